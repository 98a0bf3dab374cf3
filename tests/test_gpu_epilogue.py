"""Epilogue variants beyond the reference's V1: per-row biases (``bias1`` [H] before the
activation, ``bias2`` [N] before the final rounding, both added to the fp32 sums) and the
SiLU activation, on every kernel path -- prefill tiles (one CTA and CTA pairs), Stream-K
(the owner adds the bias once, after the partials), swap-AB decode tiles (one bias value per
feature row), fp8-weight decode tiles, hidden-resident row blocks -- against the oracle of
the same arithmetic within two output ulps plus 1e-3 * max|ref|."""
import numpy as np
import pytest
import torch

from ffn_optim_b200 import NotApplicable, prepare_ffn
from oracle import ffn_oracle as O
from tests.test_gpu_parity import assert_close_bits, bits_of

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, K, H, N, dtype): decode, ragged prefill, larger prefill
    (16, 512, 1024, 256, torch.bfloat16),
    (300, 136, 520, 200, torch.float16),
    (2048, 1024, 2048, 768, torch.bfloat16),
]


def _inputs(m, k, h, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(dtype)
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype)
    b1 = (torch.randn(h, generator=g) * 0.5).to(dtype)
    b2 = (torch.randn(n, generator=g) * 0.5).to(dtype)
    return x, w1, w2, b1, b2


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:4])) + str(s[4])[-4:])
@pytest.mark.parametrize("variant", [
    {"down_impl": "basic"}, {"down_impl": "streamk"}, {"down_impl": "full_load_a"},
    {"down_impl": "basic", "tile": "pair256x256"}, {"down_impl": "basic", "weight_format": "fp8"}],
    ids=["basic", "streamk", "full_load_a", "pair", "fp8"])
@pytest.mark.parametrize("activation,use_bias", [("gelu", True), ("silu", False), ("silu", True)])
def test_bias_and_activation_vs_oracle(shape, variant, activation, use_bias):
    m, k, h, n, dtype = shape
    x, w1, w2, b1, b2 = _inputs(m, k, h, n, dtype, m + k + h)
    kw = dict(variant, activation=activation)
    if use_bias:
        kw.update(bias1=b1.cuda(), bias2=b2.cuda())
    try:
        prepared = prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), **kw)
    except NotApplicable:
        pytest.skip("variant not applicable to this shape")
    except ValueError:
        assert variant.get("tile") == "pair256x256" and m <= 64
        pytest.skip("CTA-pair tiles are prefill tiles")
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    dt = str(dtype).removeprefix("torch.")
    f = lambda t: t.float().numpy()  # noqa: E731
    bb1, bb2 = (f(b1), f(b2)) if use_bias else (None, None)
    if variant.get("weight_format") == "fp8":
        q1 = prepared.storage[1][:, :k].cpu().numpy()
        q2 = prepared.storage[2][:, :h].cpu().numpy()
        s1, s2 = (s.cpu().numpy() for s in prepared.weight_scales)
        w1e = O.E4M3_VALUES[q1] * s1[:, None]
        w2e = O.E4M3_VALUES[q2] * s2[:, None]
        xe = O._as_fp16(f(x))
        # fp8 path: activations enter the MMA as fp16, the row scale multiplies the fp32 sum
        z = (xe @ O.E4M3_VALUES[q1].T) * s1
        if bb1 is not None:
            z = z + bb1
        hid = O.round_to(O.silu(z) if activation == "silu" else O.gelu_rational(z), dt)
        yv = (O._as_fp16(hid) @ O.E4M3_VALUES[q2].T) * s2
        if bb2 is not None:
            yv = yv + bb2
        ref = O.to_bits(yv.astype(np.float32), dt)
        del w1e, w2e
    else:
        ref = O.ffn(f(x), f(w1), f(w2), dt, staged=True, rational=True, b1=bb1, b2=bb2, activation=activation)
    assert_close_bits(bits_of(y), ref, dt)


def test_bias_validation():
    x, w1, w2, b1, b2 = _inputs(16, 64, 128, 64, torch.bfloat16, 1)
    x, w1, w2 = x.cuda(), w1.cuda(), w2.cuda()
    with pytest.raises(ValueError):
        prepare_ffn(x, w1, w2, bias1=b2.cuda())          # wrong length
    with pytest.raises(ValueError):
        prepare_ffn(x, w1, w2, bias1=b1.cuda().float())  # wrong dtype
    with pytest.raises(ValueError):
        prepare_ffn(x, w1, w2, activation="relu")
    # an unaligned view is copied into aligned storage
    buf = torch.zeros(129, dtype=torch.bfloat16, device="cuda")
    buf[1:].copy_(b1.cuda())
    y = prepare_ffn(x, w1, w2, bias1=buf[1:]).run()
    ref = prepare_ffn(x, w1, w2, bias1=b1.cuda()).run()
    assert torch.equal(y, ref)
