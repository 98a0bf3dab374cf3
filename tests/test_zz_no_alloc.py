"""The allocation-free entry point ``ffn_b200_run_noalloc``.

Some callers cannot allocate device memory while they run the FFN: an inference engine
that gives each plugin a fixed memory budget and calls it on its execution path (where a
cudaMalloc is refused or stalls every stream by synchronising the device), or a serving
loop that reserves all memory when it starts.  For them the library keeps the kernel's
scratch -- hidden activations, Stream-K partials, counters -- in a 32 MiB device array of
its own, and the caller only passes X, W1, W2 and Y.

This test calls that entry point through the C ABI twice in a row and checks each output
against the regular prepared entry point (ffn_b200_prepare / ffn_b200_run) on the same
inputs, with the tolerance of the other GPU parity tests, and against the CPU oracle (the
numpy restatement of the reference's ffn_torch): two output ulps + 1e-3*max|golden| against
the golden of the kernel's arithmetic, and the reference criterion with the max-abs bound
against the exact-erf golden.  It lives in its own file, collected last, and depends on no
state left by other tests.
"""
import ctypes

import pytest
import torch

from ffn_optim_b200 import _lib, prepare_ffn
from ffn_optim_b200.host.inputs import pitch_of
from oracle import ffn_oracle as O
from tests.test_gpu_parity import assert_close_bits, assert_criterion, bits_of

pytestmark = pytest.mark.gpu

SHAPES = [
    # (M, K, H, N, dtype, down_impl)
    (16, 4096, 16384, 4096, torch.bfloat16, "streamk"),   # decode-sized (BASELINE cfg3)
    (256, 192, 520, 136, torch.bfloat16, "streamk"),
    (512, 512, 2048, 512, torch.float16, "basic"),        # BASELINE cfg1 shape
    (6993, 104, 1000, 250, torch.float16, "full_load_a"),  # BASELINE cfg2 shape (K padded to a
                                                            # 16-byte pitch), hidden on chip
    (4096, 64, 8192, 64, torch.bfloat16, "full_load_a"),   # hidden would be 64 MiB: none needed
]


def _inputs(m, k, h, n, dtype):
    g = torch.Generator().manual_seed(m * 7 + h)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(dtype).cuda()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype).cuda()
    return x, w1, w2


def _call_noalloc(lib, prob, x, w1, w2, y, status):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.ffn_b200_run_noalloc(ctypes.byref(prob), x.data_ptr(), x.stride(0), w1.data_ptr(), w1.stride(0),
                                    w2.data_ptr(), w2.stride(0), y.data_ptr(), y.stride(0), status.data_ptr(),
                                    ctypes.c_void_p(stream))


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}x{s[2]}x{s[3]}-{s[5]}")
def test_noalloc_matches_prepared_entry_point(shape):
    m, k, h, n, dtype, down = shape
    lib = _lib.load()
    x, w1, w2 = _inputs(m, k, h, n, dtype)
    prepared = prepare_ffn(x, w1, w2, down_impl=down)
    expected = prepared.run().clone()
    prepared.check()
    dt = str(dtype).removeprefix("torch.")
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    staged = O.ffn(f(x), f(w1), f(w2), dt, staged=True, rational=True)
    golden = O.ffn(f(x), f(w1), f(w2), dt)
    prob = _lib.Problem(m, k, h, n, _lib.DTYPES[dt], _lib.DOWN_IMPL_CODES[down], 0, 0, 0)
    y = torch.full((m, pitch_of(n)), float("nan"), dtype=dtype, device="cuda")
    status = torch.full((4,), -1, dtype=torch.int32, device="cuda")
    for call in range(2):
        rc = _call_noalloc(lib, prob, x, w1, w2, y, status)
        assert rc == _lib.OK, _lib.strerror(rc)
        torch.cuda.synchronize()
        assert status.tolist()[0] == 0, (call, status.tolist())
        got = bits_of(y[:, :n])
        assert_close_bits(got, bits_of(expected), dt)
        assert_close_bits(got, staged, dt)
        assert_criterion(got, golden, dt)
        y.fill_(float("nan"))


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.load()
    m, k, h, n = 4096, 64, 8192, 64  # hidden alone is 64 MiB
    x, w1, w2 = _inputs(m, k, h, n, torch.bfloat16)
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    prob = _lib.Problem(m, k, h, n, 1, 0, 0, 0, 0)
    assert _call_noalloc(lib, prob, x, w1, w2, y, status) == _lib.ERR_SCRATCH
    assert "32 MiB" in _lib.strerror(_lib.ERR_SCRATCH)
