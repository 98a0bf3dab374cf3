"""Multi-GPU fused FFN: one process per GPU, ``torch.distributed`` over NCCL.

Two partitionings of the same FFN (the reference is single-device; these are the
multi-GPU variants of the hot path):

* **H-sharded tensor parallel** (:class:`TensorParallelFFN`): rank r holds W1 rows and W2
  columns ``[r*H/P, (r+1)*H/P)``, runs the fused kernel on its slice and produces a partial
  Y over all M rows; the partials are summed by an NCCL reduce-scatter over M (each rank
  keeps M/P rows of Y) or an all-reduce (every rank keeps Y).  M is processed in chunks so
  the collective of chunk i overlaps the kernel of chunk i+1 on NVLink.
* **M-sharded** (:class:`RowShardedFFN`): rank r holds rows ``[r*M/P, (r+1)*M/P)`` of X and
  full weights; no communication.

The slicing arithmetic (:func:`h_slice`, :func:`m_slices`, :func:`chunk_rows`,
:func:`scattered_rows`) and the collective composition (:func:`combine_partials`) are
plain functions so they can be tested with CPU ``gloo`` ranks.
"""
from __future__ import annotations

from dataclasses import dataclass


def h_slice(h: int, rank: int, world: int):
    """Hidden columns [lo, hi) owned by ``rank``: contiguous slices of whole 8-column units
    (so every boundary but H itself is a multiple of 8 and slices stay 16-byte addressable);
    sizes differ by at most one unit plus the ragged end of H (< 16 columns)."""
    units = (h + 7) // 8
    base, extra = divmod(units, world)
    lo_u = rank * base + min(rank, extra)
    hi_u = lo_u + base + (1 if rank < extra else 0)
    return min(lo_u * 8, h), min(hi_u * 8, h)


def m_slices(m: int, world: int):
    """Row ranges [lo, hi) of the M-sharded variant (sizes differ by at most one row)."""
    base, extra = divmod(m, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def chunk_rows(m: int, world: int, chunks: int):
    """Splits M into ``chunks`` pieces whose sizes are multiples of ``world`` (reduce-scatter
    needs equal shards).  Returns [(lo, hi)] or raises ValueError if M % world != 0."""
    if m % world:
        raise ValueError("reduce-scatter needs M divisible by the world size; use mode='all_reduce'")
    units = m // world
    chunks = max(1, min(chunks, units))
    base, extra = divmod(units, chunks)
    out, lo = [], 0
    for c in range(chunks):
        hi = lo + (base + (1 if c < extra else 0)) * world
        out.append((lo, hi))
        lo = hi
    return out


def scattered_rows(chunks, rank: int, world: int):
    """Global row indices a rank holds after the per-chunk reduce-scatters, in order."""
    idx = []
    for lo, hi in chunks:
        per = (hi - lo) // world
        start = lo + rank * per
        idx.extend(range(start, start + per))
    return idx


def combine_partials(partial, out, mode="reduce_scatter", group=None, async_op=False):
    """Sums the ranks' partial Y: reduce-scatter over rows into ``out`` (rows/P of them) or
    all-reduce in place (``out`` ignored).  Returns the work handle when ``async_op``."""
    import torch.distributed as dist

    if mode == "reduce_scatter":
        return dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    if mode == "all_reduce":
        return dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    raise ValueError(mode)


@dataclass
class _Chunk:
    lo: int
    hi: int
    prepared: object
    out: object


class TensorParallelFFN:
    """H-sharded fused FFN on this rank (see module docstring).

    ``x`` is the full input (replicated on every rank), ``w1``/``w2`` the full weights or
    this rank's slices (``sliced=True``).  :meth:`run` launches one fused kernel per
    M-chunk on the current stream, each followed by an asynchronous NCCL collective, and
    returns this rank's rows of Y (reduce_scatter) or the whole Y (all_reduce).
    """

    def __init__(self, x, w1, w2, *, group=None, mode="reduce_scatter", chunks=4, sliced=False,
                 down_impl="basic", block_num=None, gelu="rational", tile=None):
        import torch
        import torch.distributed as dist

        from .api import prepare_ffn

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.mode = mode
        p_shape = tuple(x.shape)
        k = p_shape[-1]
        m = x.numel() // k
        h_full = w1.shape[0] if not sliced else None
        if not sliced:
            lo, hi = h_slice(h_full, self.rank, self.world)
            w1 = w1[lo:hi]
            w2 = w2[:, lo:hi]
        # One contiguous copy of the slices, shared in place by every chunk's launch.
        w1 = w1.contiguous()
        w2 = w2.contiguous()
        self.n = w2.shape[0]
        self.m = m
        x2 = x.reshape(m, k)
        rows = chunk_rows(m, self.world, chunks) if mode == "reduce_scatter" else [(0, m)]
        self.chunks = []
        for lo, hi in rows:
            prepared = prepare_ffn(x2[lo:hi], w1, w2, down_impl=down_impl, block_num=block_num, gelu=gelu, tile=tile)
            out = None
            if mode == "reduce_scatter":
                out = torch.empty(((hi - lo) // self.world, self.n), dtype=x.dtype, device=x.device)
            self.chunks.append(_Chunk(lo, hi, prepared, out))
        self.stream = torch.cuda.current_stream()

    def launches_per_run(self):
        return len(self.chunks)

    def run(self):
        import torch

        works, partials = [], []
        for ch in self.chunks:
            y = ch.prepared.run()  # [rows, N] view of a [rows, ldy] buffer
            if y.stride(0) != self.n:
                y = y.contiguous()
            partials.append(y)
            works.append(combine_partials(y, ch.out, self.mode, self.group, async_op=True))
        for w in works:
            w.wait()
        if self.mode == "reduce_scatter":
            return torch.cat([c.out for c in self.chunks]) if len(self.chunks) > 1 else self.chunks[0].out
        return partials[0]

    def local_rows(self):
        """Global row indices of the reduce-scatter output on this rank, in output order."""
        return scattered_rows([(c.lo, c.hi) for c in self.chunks], self.rank, self.world)

    def check(self):
        for ch in self.chunks:
            ch.prepared.check()


class RowShardedFFN:
    """M-sharded fused FFN on this rank: rows ``m_slices(M, P)[rank]`` of X, full weights,
    no communication.  :meth:`run` returns this rank's rows of Y."""

    def __init__(self, x, w1, w2, *, group=None, down_impl="basic", block_num=None, gelu="rational",
                 local=False, tile=None):
        import torch.distributed as dist

        from .api import prepare_ffn

        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        k = x.shape[-1]
        m = x.numel() // k
        if local:
            x_local = x.reshape(-1, k)
            self.lo, self.hi = None, None
        else:
            self.lo, self.hi = m_slices(m, self.world)[self.rank]
            x_local = x.reshape(m, k)[self.lo:self.hi]
        self.prepared = prepare_ffn(x_local, w1, w2, down_impl=down_impl, block_num=block_num, gelu=gelu, tile=tile)

    def launches_per_run(self):
        return 1

    def run(self):
        return self.prepared.run()

    def check(self):
        self.prepared.check()
