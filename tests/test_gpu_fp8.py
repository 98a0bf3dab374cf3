"""fp8-weight decode tiles (`weight_format='fp8'`): a build extension beyond the reference.

* the device quantizer (`ffn_b200_quantize_fp8_rows`) against the oracle's e4m3 restatement,
  code for code and scale for scale;
* the fused kernel with fp8 weights against the oracle of the same arithmetic
  (`ffn_fp8_weights`: fp32 sums of fp16(x) * e4m3(code), times the row scale) within two
  output ulps plus 1e-3 * max|ref|, ragged shapes and both down implementations;
* an activation beyond the fp16 range of that MMA is reported (kernel error 6), not used;
* the BASELINE decode configuration (cfg3) against the reference's bf16 golden: e4m3 keeps
  3 mantissa bits, so each weight carries up to 2^-4 relative error and near-zero outputs
  push the reference's mean relative error (mean |d| / (|golden| + 1e-3) < 0.05, a rule for
  16-bit arithmetic) past its limit; the fp8 criterion is the relative RMS error
  ||y - golden|| / ||golden|| < 0.05, with the reference's figures reported;
* prefill shapes and full_load_a are not applicable.
"""
import numpy as np
import pytest
import torch

from ffn_optim_b200 import NotApplicable, compare, prepare_ffn, quantize_weights_fp8
from ffn_optim_b200 import cases as C
from oracle import ffn_oracle as O
from tests.test_gpu_parity import GOLDEN, assert_close_bits, bits_of

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(64, 96), (130, 1000), (7, 4096)])
def test_quantizer_matches_oracle(dtype, shape):
    rows, cols = shape
    g = torch.Generator().manual_seed(rows + cols)
    w = (torch.randn(rows, cols, generator=g) * 0.05).to(dtype)
    w[1, :] = 0
    w[2, 5] = 1e3 if dtype == torch.bfloat16 else 6e4
    codes, scales = quantize_weights_fp8(w.cuda())
    torch.cuda.synchronize()
    assert codes.shape == (rows, (cols + 15) // 16 * 16) and codes.dtype == torch.uint8
    q_ref, s_ref = O.quantize_rows_e4m3(w.float().numpy())
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(codes[:, :cols].cpu().numpy(), q_ref)


def _decode_inputs(m, k, h, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(dtype)
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype)
    return x, w1, w2


@pytest.mark.parametrize("shape", [(1, 64, 256, 128, torch.bfloat16), (16, 512, 2048, 384, torch.bfloat16),
                                   (17, 1000, 1500, 700, torch.float16), (64, 4096, 2048, 1024, torch.bfloat16),
                                   (33, 136, 520, 264, torch.float16), (5, 72, 202, 96, torch.bfloat16)],
                         ids=lambda s: "x".join(map(str, s[:4])) + str(s[4])[-4:])
@pytest.mark.parametrize("down_impl", ["basic", "streamk"])
def test_fp8_decode_vs_oracle(shape, down_impl):
    m, k, h, n, dtype = shape
    x, w1, w2 = _decode_inputs(m, k, h, n, dtype, m * 3 + k)
    try:
        prepared = prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), down_impl=down_impl, weight_format="fp8")
    except NotApplicable:
        assert down_impl == "streamk"
        pytest.skip("Stream-K not applicable")
    prepared.set_wait_limit(2.0)
    assert prepared.plan.kernel["variant"] in (10, 11)
    y = prepared.run()
    prepared.check()
    dt = str(dtype).removeprefix("torch.")
    q1 = prepared.storage[1][:, :k].cpu().numpy()
    q2 = prepared.storage[2][:, :h].cpu().numpy()
    s1, s2 = (s.cpu().numpy() for s in prepared.weight_scales)
    ref = O.ffn_fp8_weights(x.float().numpy(), q1, s1, q2, s2, dt)
    assert_close_bits(bits_of(y), ref, dt)
    first = bits_of(y)
    prepared.run()
    prepared.check()
    assert np.array_equal(bits_of(y), first)


def test_fp8_cfg3_relative_rms_vs_reference_golden():
    case = C.get_case("cfg3_bf16")
    fx = np.load(GOLDEN / "cfg3_bf16.npz")
    x, w1, w2 = C.make_inputs(case, device="cuda")
    prepared = prepare_ffn(x, w1, w2, down_impl=case["down_impl"], weight_format="fp8")
    y = prepared.run()
    prepared.check()
    got = torch.from_numpy(O.from_bits(bits_of(y), "bfloat16"))
    gold = torch.from_numpy(O.from_bits(fx["golden"], "bfloat16"))
    r = compare(got, gold)
    rel_rms = float((got - gold).norm() / gold.norm())
    print(f"fp8 cfg3 vs bf16 golden: rel_rms={rel_rms:.4f} mean_rel={r['mean_rel']:.4f} max_abs={r['max_abs']:.4g}")
    assert r["finite"] and rel_rms < 0.05, (rel_rms, r)


def test_fp8_not_applicable_to_prefill_and_full_load_a():
    x, w1, w2 = _decode_inputs(256, 64, 128, 64, torch.bfloat16, 1)
    with pytest.raises(NotApplicable):
        prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), weight_format="fp8")
    x, w1, w2 = _decode_inputs(16, 64, 128, 64, torch.bfloat16, 2)
    with pytest.raises(NotApplicable):
        prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), weight_format="fp8", down_impl="full_load_a")
    with pytest.raises(ValueError):
        prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), weight_format="fp8", tile="swap16")
    x, w1, w2 = _decode_inputs(16, 65, 128, 64, torch.bfloat16, 4)  # odd K: code pairs per TMA element
    with pytest.raises(NotApplicable):
        prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), weight_format="fp8")


def test_fp8_reports_activations_beyond_fp16():
    x, w1, w2 = _decode_inputs(16, 256, 512, 256, torch.bfloat16, 3)
    x[3, 7] = 1e6
    prepared = prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), weight_format="fp8")
    prepared.set_wait_limit(2.0)
    prepared.run()
    torch.cuda.synchronize()
    assert prepared.status()[0] == 6
    with pytest.raises(RuntimeError, match="fp16 range"):
        prepared.check()
    x[3, 7] = 1.0
    prepared.run(x.cuda())
    prepared.check()
