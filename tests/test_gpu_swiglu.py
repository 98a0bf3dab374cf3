"""SwiGLU hidden layer (``activation='swiglu'``), beyond the reference's V1:
hidden = SiLU(x W_gate^T) * (x W_up^T), y = hidden W2^T, with ``weight1 = [W_gate; W_up]``.

prepare_ffn packs W1 into the kernel's row order (``pack_swiglu``) and the epilogue forms
each hidden value from its gate and up sums in fp32 before the one rounding of hidden.  Every
tile family runs against the oracle of the same arithmetic within two output ulps plus
1e-3 * max|ref|: one-CTA prefill tiles (four and eight epilogue warps), CTA pairs, Stream-K
(the owner adds the gate and up partials), the swap-AB decode tiles with and without K-step
chains, fp8-weight decode tiles, hidden-resident row blocks (each 128-row chunk of the
packed W1 gives 64 hidden columns, one down k-block; split over clusters for few row
blocks); ragged H (a padded last 64-row block).
"""
import numpy as np
import pytest
import torch

from ffn_optim_b200 import NotApplicable, prepare_ffn
from oracle import ffn_oracle as O
from tests.test_gpu_parity import assert_close_bits, bits_of

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, K, H, N, dtype)
    (1, 256, 512, 128, torch.bfloat16),
    (16, 512, 1024, 256, torch.bfloat16),
    (50, 136, 520, 200, torch.float16),
    (300, 136, 520, 200, torch.float16),
    (2048, 1024, 2048, 768, torch.bfloat16),
]


def _inputs(m, k, h, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w1 = (torch.randn(2 * h, k, generator=g) * k ** -0.5).to(dtype)
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype)
    b2 = (torch.randn(n, generator=g) * 0.5).to(dtype)
    return x, w1, w2, b2


def _unpack(z, h, swap_ab):
    """Gate and up columns of sums over the packed W1 rows (the inverse of ``pack_swiglu``)."""
    if swap_ab:
        return z[:, 0::2][:, :h], z[:, 1::2][:, :h]
    blocks = z.shape[1] // 128
    v = z.reshape(z.shape[0], blocks, 2, 64)
    return v[:, :, 0, :].reshape(z.shape[0], -1)[:, :h], v[:, :, 1, :].reshape(z.shape[0], -1)[:, :h]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:4])) + str(s[4])[-4:])
@pytest.mark.parametrize("variant", [
    {}, {"down_impl": "streamk"}, {"tile": "cta128x128"}, {"tile": "pair256x256"}, {"tile": "swap16k4"},
    {"tile": "swap64"}, {"weight_format": "fp8"}, {"down_impl": "full_load_a"}],
    ids=["auto", "streamk", "epi8", "pair", "swap16k4", "swap64", "fp8", "full_load_a"])
def test_swiglu_vs_oracle(shape, variant):
    m, k, h, n, dtype = shape
    x, w1, w2, b2 = _inputs(m, k, h, n, dtype, m + 7 * h)
    use_b2 = m == 16 or m == 300
    kw = dict(variant, activation="swiglu")
    if use_b2:
        kw["bias2"] = b2.cuda()
    try:
        prepared = prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), **kw)
    except NotApplicable:
        pytest.skip("variant not applicable to this shape")
    except ValueError:
        assert variant.get("tile") in ("pair256x256", "cta128x128", "swap16k4", "swap64")
        pytest.skip("tile family not applicable to this M")
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    dt = str(dtype).removeprefix("torch.")
    f = lambda t: t.float().numpy()  # noqa: E731
    bb2 = f(b2) if use_b2 else None
    if variant.get("weight_format") == "fp8":
        swap = bool(prepared.plan.kernel["swap_ab"])
        q1 = prepared.storage[1][:, :k].cpu().numpy()
        q2 = prepared.storage[2][:, :h].cpu().numpy()
        s1, s2 = (s.cpu().numpy() for s in prepared.weight_scales)
        z = (O._as_fp16(f(x)) @ O.E4M3_VALUES[q1].T) * s1  # sums over the packed rows
        gate, up = _unpack(z.astype(np.float32), h, swap)
        hid = O.round_to(O.silu(gate) * up, dt)
        yv = (O._as_fp16(hid) @ O.E4M3_VALUES[q2].T) * s2
        if bb2 is not None:
            yv = yv + bb2
        ref = O.to_bits(yv.astype(np.float32), dt)
    else:
        ref = O.ffn(f(x), f(w1), f(w2), dt, staged=True, b2=bb2, activation="swiglu")
    assert_close_bits(bits_of(y), ref, dt)
    first = bits_of(y)
    prepared.run()
    prepared.check()
    assert np.array_equal(bits_of(y), first)


def test_swiglu_rejections():
    x, w1, w2, _ = _inputs(256, 64, 128, 64, torch.bfloat16, 1)
    with pytest.raises(NotApplicable):  # full_load_a keeps Y in TMEM: N <= 512
        prepare_ffn(x.cuda(), w1.cuda(), torch.zeros(600, 128, dtype=torch.bfloat16).cuda(), activation="swiglu",
                    down_impl="full_load_a")
    with pytest.raises(ValueError):  # W1 must hold 2H rows
        prepare_ffn(x.cuda(), w1[:128].cuda(), w2.cuda(), activation="swiglu")
    with pytest.raises(ValueError):
        prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), activation="swiglu", bias1=torch.zeros(128).cuda())
