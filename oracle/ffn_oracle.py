"""CPU oracle of the fused FFN -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference leg may import it.  The product path
(``ffn_optim_b200``) never imports it and has no CPU fallback.

It restates, in numpy (float32 BLAS + explicit rounding), the reference's torch golden path
``validation/reference.py`` of hxtsg/ffn_optim:

  * :func:`gelu_rational`  <- validation/reference.py:5-13 (the kernel's clipped rational erf;
    same coefficients as ops/kernel/ffn.py:556-566)
  * :func:`gelu_erf`       <- torch.nn.functional.gelu(approximate='none') as called at
    validation/reference.py:20  (0.5 z (1 + erf(z / sqrt 2)), scipy's erf)
  * :func:`ffn`            <- validation/reference.py:16-23 (fp32 X.W1^T -> GELU -> optional
    hidden rounding to the input dtype (staged) -> fp32 .W2^T -> round to the input dtype)
  * :func:`round_to`       <- the ``.to(x.dtype)`` casts: IEEE round-to-nearest-even to fp16 /
    bf16

Beyond the reference (its V1 has no quantized weights): :func:`quantize_rows_e4m3` and
:func:`ffn_fp8_weights` restate this build's fp8-weight decode path -- per-row scale
absmax/448 (IEEE fp32 division), codes RN-even with saturation to +-448 in the OCP e4m3
("fn") format, activations entering the MMA as fp16, the kernel's fp32 sum multiplied by
the row scale.

Also beyond the reference (it is single-device): :func:`round_f24` and :func:`ffn_tp_partials`
restate the arithmetic of this build's H-sharded multi-GPU path -- per-rank fp32 partials
over hidden-column slices, each rounded to the wire format (fp32, 24-bit, or the input
dtype), summed in ascending rank order, rounded once.

Pinning: ``tests/golden/`` holds outputs of the reference's own ``ffn_torch`` (imported from
the reference checkout by ``tests/golden/make_golden.py``) on the seeded inputs of each case;
``tests/test_oracle.py`` checks this restatement against them (at most one unit in the last
place of the output dtype apart, the difference between two fp32 BLAS summation orders).
"""
from __future__ import annotations

import numpy as np

SQRT1_2 = np.float32(0.70710678118654752)

_P = (0.053443748819, 7.5517016694, 101.62808918, 1393.8061484, 5063.7915060, 29639.384698)
_Q = (31.212858877, 398.56963806, 3023.1248150, 13243.365831, 26267.224157)


def gelu_rational(z):
    """Clipped rational-erf GELU in float32 (validation/reference.py:5-13).

    Evaluated with the same operation order as the reference (torch applies the Python
    float constants to float32 tensors as float32 scalars): t = clip(z/sqrt2, +-3.92),
    p = t * P(t^2), q = Q(t^2), result 0.5 z (1 + p / q).
    """
    z = np.asarray(z, dtype=np.float32)
    f = np.float32
    t = np.clip(z * SQRT1_2, f(-3.92), f(3.92))
    t2 = t * t
    p = t2 * f(_P[0]) + f(_P[1])
    for c in _P[2:]:
        p = p * t2 + f(c)
    p = p * t
    q = t2 + f(_Q[0])
    for c in _Q[1:]:
        q = q * t2 + f(c)
    return f(0.5) * z * (f(1) + p / q)


def gelu_erf(z):
    """Exact-erf GELU in float32: 0.5 z (1 + erf(z / sqrt 2))."""
    from scipy.special import erf

    z = np.asarray(z, dtype=np.float32)
    return (z * np.float32(0.5) * (np.float32(1) + erf(z * SQRT1_2).astype(np.float32))).astype(np.float32)


def bf16_bits(a):
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN stays NaN)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    nan = np.isnan(a)
    out = rounded.astype(np.uint16)
    if nan.any():
        out[nan] = np.uint16(0x7FC0)
    return out


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def to_bits(a, dtype):
    """float32 values -> uint16 bit patterns of ``dtype`` ('float16' | 'bfloat16')."""
    if dtype == "bfloat16":
        return bf16_bits(a)
    if dtype == "float16":
        return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)
    raise ValueError(dtype)


def from_bits(bits, dtype):
    """uint16 bit patterns of ``dtype`` -> float32 values."""
    if dtype == "bfloat16":
        return bf16_to_f32(bits)
    if dtype == "float16":
        return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)
    raise ValueError(dtype)


def round_to(a, dtype):
    """Rounds float32 values to ``dtype`` and returns them as float32 (the ``.to(dtype)`` cast)."""
    return from_bits(to_bits(a, dtype), dtype)


def silu(z):
    """SiLU in float32: z * sigmoid(z) = z / (1 + exp(-z)) (build extension beyond the
    reference's V1)."""
    z = np.asarray(z, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (z / (np.float32(1) + np.exp(-z))).astype(np.float32)


def ffn(x, w1, w2, dtype, *, staged=False, rational=False, b1=None, b2=None, activation="gelu"):
    """Oracle of validation/reference.py:16-23 on float32 arrays holding ``dtype`` values.

    ``x`` is [..., K] (already restricted to the rows of interest), ``w1`` [H, K],
    ``w2`` [N, H].  Returns the output's uint16 bit patterns, shape [..., N].  Build
    extensions (not in the reference): optional biases ``b1`` [H] / ``b2`` [N] added to the
    fp32 sums (before the activation / before the final rounding), ``activation='silu'``,
    and ``activation='swiglu'`` with ``w1`` = [gate rows; up rows] ([2H, K]):
    hidden = SiLU(x gate^T) * (x up^T).
    """
    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    z = x.reshape(-1, x.shape[-1]) @ np.asarray(w1, dtype=np.float32).T
    if b1 is not None:
        z = (z + np.asarray(b1, dtype=np.float32)).astype(np.float32)
    if activation == "silu":
        hidden = silu(z)
    elif activation == "swiglu":  # w1 = [gate rows; up rows], [2H, K]
        h = z.shape[1] // 2
        hidden = (silu(z[:, :h]) * z[:, h:]).astype(np.float32)
    else:
        hidden = gelu_rational(z) if rational else gelu_erf(z)
    if staged:
        hidden = round_to(hidden, dtype)
    y = hidden @ np.asarray(w2, dtype=np.float32).T
    if b2 is not None:
        y = (y + np.asarray(b2, dtype=np.float32)).astype(np.float32)
    return to_bits(y, dtype).reshape(*lead, w2.shape[0])


def ulp_distance(a_bits, b_bits):
    """Distance in representable steps between two uint16 arrays of the same 16-bit format."""
    def key(b):
        b = np.asarray(b, dtype=np.uint16).astype(np.int32)
        return np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + b)
    return np.abs(key(a_bits) - key(b_bits))


def _e4m3_table():
    """float32 value of every e4m3 code (sign | 4-bit exponent, bias 7 | 3-bit mantissa);
    0x7F / 0xFF are NaN, there are no infinities."""
    vals = np.zeros(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        e, m = (code >> 3) & 0xF, code & 0x7
        if e == 15 and m == 7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = sign * (m / 8.0) * 2.0 ** -6
        else:
            vals[code] = sign * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_VALUES = _e4m3_table()
_E4M3_POS = E4M3_VALUES[:127]  # codes 0..126: the finite non-negative values, ascending


def e4m3_codes(v):
    """float32 -> e4m3 codes: round to nearest, ties to the even code, saturate to +-448
    (the cvt.rn.satfinite.e4m3x2.f32 rule); the sign of zero is kept."""
    v = np.asarray(v, dtype=np.float32)
    a = np.minimum(np.abs(v), np.float32(448.0))
    hi = np.clip(np.searchsorted(_E4M3_POS, a, side="left"), 0, 126)
    lo = np.maximum(hi - 1, 0)
    d_lo = a - _E4M3_POS[lo]
    d_hi = _E4M3_POS[hi] - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    return np.where(np.signbit(v), code | np.uint8(0x80), code).astype(np.uint8)


def quantize_rows_e4m3(w):
    """Per-row fp8 quantization of ``w`` [rows, cols] (float32 holding fp16/bf16 values):
    returns (codes uint8 [rows, cols], scales float32 [rows])."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    scales = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    return e4m3_codes(w / scales[:, None]), scales


def _as_fp16(a):
    """Round-to-nearest-even to fp16 (subnormals kept), back to float32: the fp8-weight
    path multiplies fp16 x fp16, so 16-bit activations enter the MMA as fp16."""
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def ffn_fp8_weights(x, q1, s1, q2, s2, dtype, *, rational=True):
    """The fp8-weight path on float32 activations: z = (fp16(x) . e4m3(q1)^T) * s1, hidden =
    RN_dtype(GELU(z)), y = RN_dtype((fp16(hidden) . e4m3(q2)^T) * s2).  (fp16(.) is exact
    for bf16 values inside fp16's normal range.)  Returns uint16 bits."""
    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    w1 = E4M3_VALUES[np.asarray(q1, dtype=np.uint8)]
    w2 = E4M3_VALUES[np.asarray(q2, dtype=np.uint8)]
    z = (_as_fp16(x.reshape(-1, x.shape[-1])) @ w1.T) * np.asarray(s1, dtype=np.float32)
    hidden = round_to(gelu_rational(z) if rational else gelu_erf(z), dtype)
    y = (_as_fp16(hidden) @ w2.T) * np.asarray(s2, dtype=np.float32)
    return to_bits(y, dtype).reshape(*lead, w2.shape[0])


def round_f24(a):
    """fp32 values rounded to nearest (ties to even) at bit 8 of the word, the low 8 bits
    cleared: sign, exponent and 15 explicit mantissa bits -- the 24-bit partial format of the
    fused reduce-scatter (``partial='fp24'``; build extension).  Relative error <= 2^-16."""
    b = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (b + 0x7F + ((b >> 8) & 1)) & 0xFFFFFF00
    return r.astype(np.uint32).view(np.float32)


def ffn_tp_partials(x, w1, w2, dtype, slices, partial="fp32", *, rational=True):
    """H-sharded FFN on len(slices) ranks: rank r's fp32 partial Y over hidden columns
    ``slices[r] = (lo, hi)`` (GELU of the fp32 up sum, hidden rounded to ``dtype``), rounded
    to the wire format ``partial`` ('fp32' | 'fp24' | 'input'), the partials summed in fp32 in
    ascending rank order, then rounded once to ``dtype``.  Returns uint16 bit patterns."""
    x = np.asarray(x, dtype=np.float32)
    w1 = np.asarray(w1, dtype=np.float32)
    w2 = np.asarray(w2, dtype=np.float32)
    acc = None
    for lo, hi in slices:
        z = x @ w1[lo:hi].T
        hidden = round_to(gelu_rational(z) if rational else gelu_erf(z), dtype)
        part = (hidden @ w2[:, lo:hi].T).astype(np.float32)
        if partial == "fp24":
            part = round_f24(part)
        elif partial == "input":
            part = round_to(part, dtype)
        elif partial != "fp32":
            raise ValueError(partial)
        acc = part if acc is None else (acc + part).astype(np.float32)
    return to_bits(acc, dtype)
