"""Case schema and deterministic seeded inputs (mirrors common/cases.py of the reference).

Schema v1 of the reference (case_id, shape, weight1_shape, weight2_shape, dtype, layout,
seed, noncontiguous) with three optional additions used by the BASELINE configurations:

  * ``distribution``: 'normal_fanin' (default; X ~ N(0,1), W ~ N(0,1) / sqrt(fan_in), as
    common/cases.py:34-50) or 'uniform2_normal005' (X ~ U(-2,2), W ~ N(0, 0.05^2));
  * ``x_view``: 'transpose_last2' builds X as the transposed view of a tensor whose last
    two dims are swapped (a non-contiguous, non-collapsible X);
  * ``down_impl``: the down-projection implementation the configuration is quoted with.

Values come from numpy's PCG64 generator (platform independent): X, W1 and W2 each have
their own stream (children of ``SeedSequence(seed)``), X one child stream per block of
4096 rows, so weights and any X row subset regenerate bit-identically on every machine.
Values are drawn in float32 and rounded to nearest even into the case dtype.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

from .host.inputs import problem_from_shapes

CASES_FILE = Path(__file__).resolve().parent / "configs" / "cases.json"


def load_cases(path=CASES_FILE):
    data = json.loads(Path(path).read_text())
    if not isinstance(data, dict) or data.get("schema_version") != 1:
        raise ValueError("Expected case schema_version=1")
    cases = data.get("cases")
    if not isinstance(cases, list) or not cases:
        raise ValueError("cases must be a non-empty list")
    seen = set()
    for case in cases:
        name = case.get("case_id")
        if not isinstance(name, str) or not name or name in seen:
            raise ValueError("case_id must be a unique non-empty string")
        seen.add(name)
        case_problem(case)
        if type(case.get("seed", 0)) is not int:
            raise ValueError("seed must be an integer")
        if type(case.get("noncontiguous", False)) is not bool:
            raise ValueError("noncontiguous must be boolean")
        if case.get("distribution", "normal_fanin") not in ("normal_fanin", "uniform2_normal005"):
            raise ValueError("unknown distribution")
        if case.get("x_view", "plain") not in ("plain", "transpose_last2"):
            raise ValueError("unknown x_view")
    return cases


def get_case(case_id, path=CASES_FILE):
    for case in load_cases(path):
        if case["case_id"] == case_id:
            return case
    raise KeyError(case_id)


def case_problem(case):
    return problem_from_shapes(case["shape"], case["weight1_shape"], case["weight2_shape"],
                               case["dtype"], case.get("layout", "linear"))


def _round_bits(a, dtype):
    if dtype == "float16":
        return a.astype(np.float16).view(np.uint16)
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


X_BLOCK_ROWS = 4096


def _streams(case):
    """Independent generators for X, W1 and W2 (numpy SeedSequence children 0, 1, 2)."""
    return np.random.SeedSequence(case.get("seed", 0)).spawn(3)


def _x_gen_shape(case):
    p = case_problem(case)
    shape = list(p.input_shape)
    if case.get("x_view", "plain") == "transpose_last2":
        shape[-1], shape[-2] = shape[-2], shape[-1]
    return shape


def _draw(rng, shape, dist, scale):
    if dist == "normal_fanin":
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
    return rng.uniform(-2.0, 2.0, shape).astype(np.float32)


def x_rows(case, start, stop):
    """Bit patterns of rows [start, stop) of X in generation layout (flattened leading dims).

    Row block b (X_BLOCK_ROWS rows) is drawn from its own child stream, so any subset of
    rows is reproducible without drawing the rest of X.
    """
    p = case_problem(case)
    shape = _x_gen_shape(case)
    cols = shape[-1]
    rows_total = int(np.prod(shape[:-1]))
    dist = case.get("distribution", "normal_fanin")
    ss_x = _streams(case)[0]
    nblocks = (rows_total + X_BLOCK_ROWS - 1) // X_BLOCK_ROWS
    children = ss_x.spawn(nblocks)
    out = np.empty((stop - start, cols), dtype=np.uint16)
    b0, b1 = start // X_BLOCK_ROWS, (stop - 1) // X_BLOCK_ROWS
    for b in range(b0, b1 + 1):
        lo = b * X_BLOCK_ROWS
        hi = min(lo + X_BLOCK_ROWS, rows_total)
        rng = np.random.Generator(np.random.PCG64(children[b]))
        block = _round_bits(_draw(rng, (hi - lo, cols), dist, 1.0), p.dtype)
        s0, s1 = max(start, lo), min(stop, hi)
        out[s0 - start:s1 - start] = block[s0 - lo:s1 - lo]
    return out


def _weight_bits(seed_seq, shape, dist, scale, dtype, chunk_rows=1024):
    """One weight tensor from its own PCG64 stream, drawn in row chunks (the stream advances
    exactly as in one call, so the values are the same) and rounded chunk by chunk."""
    rng = np.random.Generator(np.random.PCG64(seed_seq))
    out = np.empty(shape, dtype=np.uint16)
    for r0 in range(0, shape[0], chunk_rows):
        rows = min(chunk_rows, shape[0] - r0)
        a = rng.standard_normal((rows, shape[1]), dtype=np.float32)
        a *= np.float32(scale)
        if dtype == "float16":
            out[r0:r0 + rows] = a.astype(np.float16).view(np.uint16)
        else:  # round to nearest even in place: u + 0x7FFF + ((u >> 16) & 1), then >> 16
            u = a.view(np.uint32)
            t = u >> np.uint32(16)
            t &= np.uint32(1)
            t += np.uint32(0x7FFF)
            u += t
            u >>= np.uint32(16)
            out[r0:r0 + rows] = u
    return out


def weights(case):
    """Bit patterns of W1 [H, K] and W2 [N, H] (drawn on two threads: independent streams)."""
    from concurrent.futures import ThreadPoolExecutor

    p = case_problem(case)
    dist = case.get("distribution", "normal_fanin")
    _, s1, s2 = _streams(case)
    if dist == "normal_fanin":
        scales = (p.k ** -0.5, p.h ** -0.5)
    else:
        scales = (0.05, 0.05)
    with ThreadPoolExecutor(2) as ex:
        f1 = ex.submit(_weight_bits, s1, (p.h, p.k), dist, scales[0], p.dtype)
        f2 = ex.submit(_weight_bits, s2, (p.n, p.h), dist, scales[1], p.dtype)
        return f1.result(), f2.result()


def make_arrays(case):
    """Returns the uint16 bit patterns (x in generation layout, w1, w2)."""
    shape = _x_gen_shape(case)
    rows_total = int(np.prod(shape[:-1]))
    x = x_rows(case, 0, rows_total).reshape(shape)
    w1, w2 = weights(case)
    return x, w1, w2


def logical_x_rows(case, rows):
    """Bit patterns [len(rows), K] of rows of the logical X (after the case's view and
    stride), regenerating only the 4096-row blocks the rows fall in when X is plain."""
    p = case_problem(case)
    if case.get("x_view", "plain") == "transpose_last2" or case.get("noncontiguous", False):
        import torch

        x, _, _ = make_inputs(case)
        flat = x.reshape(p.m, p.k).contiguous().view(torch.int16).numpy().view(np.uint16)
        return flat[np.asarray(rows)]
    blocks = {}
    out = np.empty((len(rows), p.k), dtype=np.uint16)
    for i, r in enumerate(rows):
        b = int(r) // X_BLOCK_ROWS
        if b not in blocks:
            lo = b * X_BLOCK_ROWS
            blocks[b] = (lo, x_rows(case, lo, min(lo + X_BLOCK_ROWS, p.m)))
        lo, blk = blocks[b]
        out[i] = blk[int(r) - lo]
    return out


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def make_inputs(case, device="cpu"):
    """Seeded (x, w1, w2) torch tensors with the case's dtype, shape and view."""
    import torch

    p = case_problem(case)
    dtype = getattr(torch, p.dtype)
    xb, w1b, w2b = make_arrays(case)

    def tensor(bits):
        return torch.from_numpy(bits.view(np.int16)).view(dtype).to(device)

    x, w1, w2 = tensor(xb), tensor(w1b), tensor(w2b)
    if case.get("x_view", "plain") == "transpose_last2":
        x = x.transpose(-1, -2)
    if case.get("noncontiguous", False):
        def strided(t):
            buf = torch.empty((*t.shape[:-1], t.shape[-1] * 2), dtype=t.dtype, device=t.device)
            buf[..., ::2].copy_(t)
            return buf[..., ::2]
        x, w1, w2 = map(strided, (x, w1, w2))
    return x, w1, w2


def reference_stream_inputs(case, device="cpu"):
    """(x, w1, w2) drawn exactly as the reference draws its smoke-case inputs
    (common/cases.py:34-50): one CPU ``torch.Generator`` seeded with the case's seed, standard
    normal draws for X (the input shape), then W1 [H, K] scaled by K**-0.5, then W2 [N, H]
    scaled by H**-0.5, each rounded to the case's dtype; ``noncontiguous`` cases get the same
    stride-2 views.  The draws are sequential over whole tensors, so this form is for the
    small smoke cases; the BASELINE configurations use :func:`make_inputs` (row-addressable
    streams)."""
    import torch

    p = case_problem(case)
    gen = torch.Generator(device="cpu").manual_seed(case.get("seed", 0))
    dtype = getattr(torch, p.dtype)

    def sample(shape, scale=1.0):
        return (torch.randn(shape, generator=gen) * scale).to(dtype).to(device)

    x = sample(p.input_shape)
    w1 = sample((p.h, p.k), p.k ** -0.5)
    w2 = sample((p.n, p.h), p.h ** -0.5)
    if case.get("noncontiguous", False):
        def strided(t):
            buf = torch.empty((*t.shape[:-1], t.shape[-1] * 2), dtype=t.dtype, device=t.device)
            buf[..., ::2].copy_(t)
            return buf[..., ::2]
        x, w1, w2 = map(strided, (x, w1, w2))
    return x, w1, w2
