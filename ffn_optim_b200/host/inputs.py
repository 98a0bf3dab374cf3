"""Input contract shared by the oracle, planning and device execution.

Mirrors ops/host/inputs.py of the reference: same ``Problem`` fields, same shape rules
(rank 2-8, fp16/bf16, layout='linear', max(K,H,N) <= 65535, M <= 2**31-16) and the same
exception types and messages' meaning.
"""
from __future__ import annotations

from dataclasses import dataclass
from math import prod


@dataclass(frozen=True)
class Problem:
    """Logical FFN shape (reference ops/host/inputs.py:6-26).

    ``input_shape`` is X's shape (2-8 dims, K last), ``m`` the product of its leading dims,
    ``k/h/n`` the input, hidden and output widths, ``dtype`` 'float16' or 'bfloat16'.
    Build it with :func:`problem_from_shapes`, which validates; direct construction does not.
    """

    input_shape: tuple
    m: int
    k: int
    h: int
    n: int
    dtype: str
    layout: str

    @property
    def output_shape(self):
        return (*self.input_shape[:-1], self.n)


def _shape(value, name, ranks):
    result = tuple(value)
    if len(result) not in ranks:
        raise ValueError(f"{name}: unsupported rank {len(result)}")
    if any(type(d) is not int or d <= 0 for d in result):
        raise ValueError(f"{name}: dimensions must be positive integers")
    return result


def problem_from_shapes(x_shape, w1_shape, w2_shape, dtype="float16", layout="linear"):
    """Validates shapes (reference ops/host/inputs.py:38-53) and returns a :class:`Problem`."""
    x = _shape(x_shape, "x", range(2, 9))
    w1 = _shape(w1_shape, "weight1", (2,))
    w2 = _shape(w2_shape, "weight2", (2,))
    if dtype not in ("float16", "bfloat16"):
        raise ValueError("dtype must be float16 or bfloat16")
    if layout != "linear":
        raise ValueError("Only explicit layout='linear' is supported")
    h, k = w1
    n, h2 = w2
    if x[-1] != k or h != h2:
        raise ValueError("Expected x[..., K], weight1[H,K], weight2[N,H]")
    if max(k, h, n) > 65535 or prod(x[:-1]) > 2**31 - 16:
        raise ValueError("Shape exceeds the supported bounds (max(K,H,N) <= 65535, M <= 2**31-16)")
    return Problem(x, prod(x[:-1]), k, h, n, dtype, layout)


def validate_tensors(x, weight1, weight2, layout="linear", require_cuda=False):
    """Tensor checks of reference ops/host/inputs.py:56-71, with CUDA in place of NPU."""
    import torch

    tensors = (x, weight1, weight2)
    if any(not isinstance(t, torch.Tensor) for t in tensors):
        raise TypeError("x, weight1 and weight2 must be torch.Tensor")
    if any(t.dtype != x.dtype or t.device != x.device for t in tensors):
        raise ValueError("All tensors must have the same dtype and device")
    if any(t.layout != torch.strided for t in tensors):
        raise ValueError("Only dense strided tensors are supported")
    if any(t.requires_grad for t in tensors):
        raise ValueError("Inference-only operator; detach inputs explicitly")
    if require_cuda and x.device.type != "cuda":
        raise ValueError("FFN execution requires CUDA tensors; no CPU fallback is used")
    return problem_from_shapes(x.shape, weight1.shape, weight2.shape,
                               str(x.dtype).removeprefix("torch."), layout)


def pitch_of(cols: int) -> int:
    """Row pitch in elements for a TMA-addressable row: a multiple of 8 (16 bytes)."""
    return (cols + 7) // 8 * 8


def _tma_ready(t, rows, cols):
    """True when ``t`` is a [rows, cols] view the kernel can read in place."""
    return (t.dim() == 2 and t.shape[0] == rows and t.shape[1] == cols and t.stride(1) == 1
            and t.stride(0) % 8 == 0 and t.stride(0) >= cols and t.data_ptr() % 16 == 0)


def _packed(t, rows, cols):
    """Copies ``t`` into a fresh [rows, pitch] buffer; only the first ``cols`` columns are set."""
    import torch

    buf = torch.empty((rows, pitch_of(cols)), dtype=t.dtype, device=t.device)
    buf[:, :cols].copy_(t.reshape(rows, cols))
    return buf


def pack_swiglu(weight1, hidden, swap_ab):
    """W1 = [gate rows; up rows] ([2H, K]) in the fused kernel's SwiGLU order: with
    ``swap_ab`` (decode tiles) gate row i at row 2i and up row i at 2i + 1; otherwise blocks
    of 64 gate rows each followed by the matching 64 up rows, zero rows padding the last block
    (``ffn_b200_swiglu_rows`` gives the row count)."""
    import torch

    from .. import _lib

    gate, up = weight1[:hidden], weight1[hidden:]
    k = weight1.shape[1]
    rows = int(_lib.load().ffn_b200_swiglu_rows(hidden, 1 if swap_ab else 0))
    packed = torch.zeros((rows, pitch_of(k)), dtype=weight1.dtype, device=weight1.device)
    if swap_ab:
        packed[0::2, :k] = gate
        packed[1::2, :k] = up
    else:
        blocks = rows // 128
        view = packed.view(blocks, 2, 64, packed.shape[1])
        g = torch.zeros((blocks * 64, k), dtype=weight1.dtype, device=weight1.device)
        u = torch.zeros_like(g)
        g[:hidden], u[:hidden] = gate, up
        view[:, 0, :, :k] = g.view(blocks, 64, k)
        view[:, 1, :, :k] = u.view(blocks, 64, k)
    return packed[:, :k]


def quantize_weights_fp8(weight):
    """fp8 weights for the decode tiles: ``weight`` [rows, cols] (fp16/bf16, CUDA) becomes
    ``(codes, scales)``: uint8 e4m3 codes [rows, pitch] (pitch = cols rounded up to 16
    bytes, the TMA rule for 1-byte elements) and fp32 row scales [rows], with
    ``weight[r, c] ~= e4m3(codes[r, c]) * scales[r]`` (per-row absmax / 448, RN-even,
    saturating; computed on the device by ``ffn_b200_quantize_fp8_rows``)."""
    import ctypes

    import torch

    from .. import _lib

    rows, cols = weight.shape
    src = weight if _tma_ready(weight, rows, cols) else _packed(weight.contiguous(), rows, cols)
    codes = torch.zeros((rows, (cols + 15) // 16 * 16), dtype=torch.uint8, device=weight.device)
    scales = torch.empty(rows, dtype=torch.float32, device=weight.device)
    dtype = str(weight.dtype).removeprefix("torch.")
    rc = _lib.load().ffn_b200_quantize_fp8_rows(src.data_ptr(), src.stride(0), _lib.DTYPES[dtype], rows, cols,
                                                codes.data_ptr(), codes.stride(0), scales.data_ptr(),
                                                ctypes.c_void_p(torch.cuda.current_stream(weight.device).cuda_stream))
    if rc != _lib.OK:
        raise ValueError(f"ffn_b200_quantize_fp8_rows: {_lib.strerror(rc)}")
    return codes, scales


def prepare_storage(x, weight1, weight2, plan):
    """Device storage for one prepared FFN (reference ops/host/inputs.py:74-90).

    The reference zero-pads every operand to its tile grid.  Here the kernels mask ragged
    edges with TMA out-of-bounds fill, so nothing is padded with zeros; an operand is only
    copied when its rows are not 16-byte addressable (non-contiguous, or K/H not a multiple
    of 8).  X is always copied into storage owned by the prepared FFN, as in the reference;
    weights that are already addressable are used in place.  Returns
    ``(x2d, w1, w2, hidden, out, workspace, counters, flags, status)``: x2d [M, ldx],
    hidden [M, ldh] (for full_load_a only [M, 8]: the hidden tensor stays on chip) and
    out [M, ldy] with 16-byte pitches, fp32 workspace and u32/i32 synchronisation words
    (zeroed).
    """
    import torch

    p = plan.problem
    dev = x.device
    xs = x.reshape(p.m, p.k) if x.is_contiguous() else x.contiguous().view(p.m, p.k)
    x2d = _packed(xs, p.m, p.k)
    # (fp8 weights arrive here as uint8 code views with 16-byte pitches: used in place)
    r1 = weight1.shape[0]  # H, or the gate/up-packed rows of a SwiGLU problem
    w1 = weight1 if _tma_ready(weight1, r1, p.k) else _packed(weight1.contiguous(), r1, p.k)
    w2 = weight2 if _tma_ready(weight2, p.n, p.h) else _packed(weight2.contiguous(), p.n, p.h)
    # full_load_a keeps the hidden row block on chip: an 8-column stand-in keeps the
    # storage tuple's shape contract (row-indexable) without the M x H buffer.
    on_chip = plan.selection.down_impl == "full_load_a"
    hidden = torch.empty((p.m, 8 if on_chip else pitch_of(p.h)), dtype=x.dtype, device=dev)
    out = torch.empty((p.m, pitch_of(p.n)), dtype=x.dtype, device=dev)
    info = plan.kernel
    ws = torch.empty(max(int(info["workspace_floats"]), 4), dtype=torch.float32, device=dev)
    counters = torch.zeros(max(int(info["counter_words"]), 1), dtype=torch.int32, device=dev)
    flags = torch.zeros(max(int(info["flag_words"]), 1), dtype=torch.int32, device=dev)
    status = torch.zeros(max(int(info["status_words"]), 4), dtype=torch.int32, device=dev)
    return x2d, w1, w2, hidden, out, ws, counters, flags, status
