"""Hidden-slice decode kernel (M <= 16 tokens; clusters of 2-8 CTAs, each CTA owning 128
hidden rows, the cluster's hidden slice exchanged in shared memory and Y reduced over the
clusters) against the oracle of the same arithmetic (fp32 sums, activation of the fp32
sum, hidden rounded once, one rounding of Y) within two output ulps plus 1e-3 * max|ref|:
ragged K/H/N, hidden blocks beyond H, several super-blocks per cluster, every activation,
biases, fp16 and bf16, run-to-run bit identity, and the automatic choice for cfg3."""
import numpy as np
import pytest
import torch

from ffn_optim_b200 import cases as C
from ffn_optim_b200 import prepare_ffn
from oracle import ffn_oracle as O
from tests.test_gpu_parity import GOLDEN, assert_close_bits, assert_criterion, bits_of

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, K, H, N, dtype, activation, bias)
    (1, 64, 128, 64, torch.bfloat16, "gelu", False),        # one hidden block: 7 CTAs of zero rows
    (5, 200, 1000, 300, torch.float16, "gelu", False),      # ragged K, H, N
    (16, 520, 2100, 1100, torch.bfloat16, "gelu", True),    # biases; N not a multiple of 128 * 8
    (9, 1024, 3000, 520, torch.float16, "silu", False),
    (16, 256, 8192, 4096, torch.bfloat16, "gelu", False),   # 8 super-blocks, 32 n-blocks
    (3, 136, 40000, 200, torch.bfloat16, "gelu", True),     # 40 super-blocks: several per cluster
    (16, 4096, 16384, 4096, torch.bfloat16, "erf", False),  # the cfg3 shape, exact-erf GELU
]


def _inputs(m, k, h, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(dtype)
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype)
    b1 = (torch.randn(h, generator=g) * 0.5).to(dtype)
    b2 = (torch.randn(n, generator=g) * 0.5).to(dtype)
    return x, w1, w2, b1, b2


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:4])) + str(s[4])[-4:] + s[5])
def test_hslice_vs_oracle(shape):
    m, k, h, n, dtype, act, use_bias = shape
    x, w1, w2, b1, b2 = _inputs(m, k, h, n, dtype, m * 7 + h)
    kw = dict(tile="hslice16", down_impl="basic")
    if act == "erf":
        kw["gelu"] = "erf"
    else:
        kw["activation"] = act
    if use_bias:
        kw.update(bias1=b1.cuda(), bias2=b2.cuda())
    prepared = prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), **kw)
    assert prepared.plan.kernel["variant"] == 12 and prepared.plan.kernel["row_split"] in (2, 4, 8)
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    dt = str(dtype).removeprefix("torch.")
    f = lambda t: t.float().numpy()  # noqa: E731
    bb1, bb2 = (f(b1), f(b2)) if use_bias else (None, None)
    ref = O.ffn(f(x), f(w1), f(w2), dt, staged=True, rational=act != "erf", b1=bb1, b2=bb2,
                activation="silu" if act == "silu" else "gelu")
    got = bits_of(y)
    assert_close_bits(got, ref, dt)
    for _ in range(2):  # fixed summation order: identical bits on every run
        prepared.run()
        prepared.check()
        assert np.array_equal(bits_of(y), got)


@pytest.mark.parametrize("down_impl", ["streamk", "basic"])
def test_cfg3_uses_hslice_and_matches_golden(down_impl):
    case = C.get_case("cfg3_bf16")
    fx = np.load(GOLDEN / "cfg3_bf16.npz")
    x, w1, w2 = C.make_inputs(case, device="cuda")
    prepared = prepare_ffn(x, w1, w2, down_impl=down_impl)
    assert prepared.plan.kernel["variant"] == 12 and prepared.plan.block_num == 128
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    got = bits_of(y)
    assert_close_bits(got, fx["staged_rational"], "bfloat16")
    assert_criterion(got, fx["golden"], "bfloat16")
    # the two-phase swap-AB kernel on the same inputs agrees within the same bound
    other = prepare_ffn(x, w1, w2, down_impl=down_impl, tile="swap16")
    other.set_wait_limit(2.0)
    y2 = other.run()
    other.check()
    assert_close_bits(bits_of(y2), fx["staged_rational"], "bfloat16")


def test_hslice_graph_and_host_path():
    """Captured in a CUDA graph and replayed, and through run_host (pinned host buffers)."""
    x, w1, w2, _, _ = _inputs(16, 512, 4096, 1024, torch.bfloat16, 3)
    prepared = prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), tile="hslice16")
    prepared.set_wait_limit(2.0)
    y = prepared.run().clone()
    prepared.check()
    graph = prepared.capture_graph()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    prepared.check()
    assert torch.equal(prepared.storage[4][:, :1024], y)
    xh = x.pin_memory()
    yh = torch.empty((16, 1024), dtype=torch.bfloat16).pin_memory()
    prepared.run_host(xh, yh)
    assert torch.equal(yh, y.cpu())
