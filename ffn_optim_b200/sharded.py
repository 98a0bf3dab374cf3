"""Multi-GPU fused FFN: one process per GPU, ``torch.distributed`` over NCCL.

Two partitionings of the same FFN (the reference is single-device; these are the
multi-GPU variants of the hot path):

* **H-sharded tensor parallel** (:class:`TensorParallelFFN`): rank r holds W1 rows and W2
  columns ``[r*H/P, (r+1)*H/P)``, runs the fused kernel on its slice and produces a partial
  Y over all M rows; the partials are summed by an NCCL reduce-scatter over M (each rank
  keeps M/P rows of Y) or an all-reduce (every rank keeps Y).  M is processed in chunks so
  the collective of chunk i overlaps the kernel of chunk i+1 on NVLink.
* **H-sharded with the reduce-scatter fused into the kernel**
  (:class:`FusedTensorParallelFFN`): no NCCL call; the kernel's down-phase epilogue pushes
  partial tiles to their owning GPU over NVLink and owners reduce them.
* **M-sharded** (:class:`RowShardedFFN`): rank r holds rows ``[r*M/P, (r+1)*M/P)`` of X and
  full weights; no communication.

The slicing arithmetic (:func:`h_slice`, :func:`m_slices`, :func:`chunk_rows`,
:func:`scattered_rows`) and the collective composition (:func:`combine_partials`) are
plain functions so they can be tested with CPU ``gloo`` ranks.
"""
from __future__ import annotations

import ctypes
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
                 down_impl="basic", block_num=None, gelu="rational", tile=None, reserve_sms=16):
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
        # The fused kernel is persistent (one CTA per SM); leaving `reserve_sms` SMs free lets
        # NCCL's collective kernels run beside it, so chunk i's reduce-scatter overlaps the
        # kernel of chunk i+1 instead of waiting for it.
        if block_num is None and reserve_sms:
            block_num = torch.cuda.get_device_properties(x.device).multi_processor_count - int(reserve_sms)
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
                 local=False, tile=None, schedule=None):
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
        self.prepared = prepare_ffn(x_local, w1, w2, down_impl=down_impl, block_num=block_num, gelu=gelu, tile=tile,
                                    schedule=schedule)

    def launches_per_run(self):
        return 1

    def run(self):
        return self.prepared.run()

    def run_host(self, x_host, y_host, chunks=8):
        """This rank's rows from host memory to host memory (``PreparedFFN.run_host``):
        ``x_host`` [rows, K] and ``y_host`` [rows, N] are pinned CPU tensors of this rank's
        ``m_slices`` rows; copies overlap the kernels of other row chunks."""
        return self.prepared.run_host(x_host, y_host, chunks=chunks)

    def check(self):
        self.prepared.check()


def band_order(world: int, rank: int):
    """Order in which ``rank`` visits the down phase's row bands under the fused
    reduce-scatter: the other ranks' bands first (starting with the next rank), its own last."""
    return [(rank + 1 + i) % world for i in range(world)]


class FusedTensorParallelFFN:
    """H-sharded fused FFN whose reduce-scatter runs inside the kernel, over NVLink.

    Same partitioning as :class:`TensorParallelFFN` (rank r holds W1 rows / W2 columns of
    ``h_slice(H, r, P)``), but no NCCL call: during the down phase each rank pushes the
    partial of every tile outside its own M/P-row band straight into the owning rank's
    staging buffer (peer bulk stores, then a system-scope release), and each rank sums the P
    partials of its own band in ascending rank order and stores its Y rows.  ``partial``
    selects what crosses NVLink: ``'fp32'`` (default; the owner sums unrounded partials, so
    every output keeps the single-GPU error bound), ``'fp24'`` (fp32 rounded to nearest at
    24 bits -- sign, exponent, 15 mantissa bits -- sent as a 16-bit and an 8-bit plane: 3/4
    of the fp32 bytes, a relative error below 2^-16 per partial) or ``'input'`` (partials
    rounded to the input dtype: half the NVLink bytes, up to P-1 extra roundings per output).  Staging and
    push-count buffers are CUDA IPC buffers exchanged once at construction.  :meth:`run`
    launches one kernel and returns this rank's rows ``local_rows()`` of Y.

    :meth:`close` is collective: every rank calls it together (it synchronises and meets the
    other ranks before releasing memory that their kernels write into).
    """

    def __init__(self, x, w1, w2, *, group=None, sliced=False, down_impl="basic", block_num=None,
                 gelu="rational", tile="cta128x256", partial="fp32"):
        import torch
        import torch.distributed as dist

        from . import _lib
        from .api import prepare_ffn
        from .host.inputs import pitch_of

        if partial not in _lib.PARTIAL_TYPES:
            raise ValueError(f"partial must be one of {sorted(_lib.PARTIAL_TYPES)}")
        self.partial = partial
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._own, self._opened, self._closed = [], [], False
        k = x.shape[-1]
        m = x.numel() // k
        if not sliced:
            lo, hi = h_slice(w1.shape[0], self.rank, self.world)
            w1, w2 = w1[lo:hi], w2[:, lo:hi]
        w1, w2 = w1.contiguous(), w2.contiguous()
        self.m, self.n = m, w2.shape[0]
        self.prepared = prepare_ffn(x.reshape(m, k), w1, w2, down_impl=down_impl, block_num=block_num, gelu=gelu,
                                    tile=tile)
        lib = _lib.load()
        h = self.prepared.handle
        code = _lib.PARTIAL_TYPES[partial]
        sb, fb = ctypes.c_uint64(), ctypes.c_uint64()
        if lib.ffn_b200_reduce_scatter_bytes(h, self.world, code, ctypes.byref(sb), ctypes.byref(fb)) != _lib.OK:
            raise ValueError("fused reduce-scatter needs M divisible by world*tile rows and a one-CTA prefill tile")
        handles = []
        with torch.cuda.device(x.device):
            for size in (sb.value, fb.value):
                ptr, ipc = ctypes.c_void_p(), (ctypes.c_char * 64)()
                rc = lib.ffn_b200_peer_alloc(size, ctypes.byref(ptr), ipc)
                if rc != _lib.OK:
                    raise RuntimeError(f"ffn_b200_peer_alloc: {_lib.strerror(rc)}")
                self._own.append(ptr)
                handles.append(bytes(ipc))
            everyone = [None] * self.world
            dist.all_gather_object(everyone, handles, group=group)
            stage = (ctypes.c_void_p * self.world)()
            flags = (ctypes.c_void_p * self.world)()
            for r in range(self.world):
                if r == self.rank:
                    stage[r], flags[r] = self._own[0], self._own[1]
                    continue
                ptrs = []
                for blob in everyone[r]:
                    ptr = ctypes.c_void_p()
                    rc = lib.ffn_b200_peer_open((ctypes.c_char * 64).from_buffer_copy(blob), ctypes.byref(ptr))
                    if rc != _lib.OK:
                        raise RuntimeError(f"ffn_b200_peer_open: {_lib.strerror(rc)}")
                    self._opened.append(ptr)
                    ptrs.append(ptr)
                stage[r], flags[r] = ptrs
            self.y = torch.empty((m // self.world, pitch_of(self.n)), dtype=x.dtype, device=x.device)
            rc = lib.ffn_b200_set_reduce_scatter(h, self.world, self.rank, code, stage, flags, self.y.data_ptr(),
                                                 self.y.stride(0))
            if rc != _lib.OK:
                raise ValueError(f"ffn_b200_set_reduce_scatter: {_lib.strerror(rc)}")
            torch.cuda.synchronize()
        dist.barrier(group=group)  # every rank has mapped every buffer before anyone pushes

    def launches_per_run(self):
        return 1

    def run(self):
        if self._closed:
            raise RuntimeError("FusedTensorParallelFFN has been closed")
        self.prepared.run()
        return self.y[:, :self.n]

    def collective_reset(self):
        """Every rank clears its push counts and restarts its launch epoch, at a point where
        no rank has a kernel in flight (all ranks call this together)."""
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.prepared.reset()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def local_rows(self):
        per = self.m // self.world
        return list(range(self.rank * per, (self.rank + 1) * per))

    def check(self):
        self.prepared.check()

    def close(self):
        """Releases the peer mappings and this rank's staging buffers.  Collective: every rank
        calls it at the same point.  This rank's kernels are complete (synchronize) and every
        other rank's are too (barrier) before any buffer a peer kernel writes into is freed,
        so no GPU ever stores into freed memory, even after a launch that timed out."""
        import torch
        import torch.distributed as dist

        from . import _lib

        if self._closed:
            return
        with torch.cuda.device(self.y.device):
            torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self._release(_lib.load())

    def _release(self, lib):
        for ptr in self._opened:
            lib.ffn_b200_peer_close(ptr)
        for ptr in self._own:
            lib.ffn_b200_peer_free(ptr)
        self._opened, self._own, self._closed = [], [], True

    def __del__(self):
        # Without the collective close() no rank can know that the other GPUs have stopped
        # writing into this rank's staging buffers, so they are left allocated (leaked until
        # the process exits) rather than freed under a peer's stores.
        if not getattr(self, "_closed", True) and getattr(self, "_own", None):
            import warnings

            warnings.warn("FusedTensorParallelFFN dropped without close(): peer-visible buffers are leaked",
                          ResourceWarning, stacklevel=2)


def tp_dp_groups(world: int, tp: int):
    """Rank lists of the tensor-parallel groups of a ``tp`` x ``world/tp`` layout: ranks
    [g*tp, (g+1)*tp) form group g (neighbouring ranks, so a group's peers share the node's
    NVSwitch like any others).  Raises ValueError unless 2 <= tp <= world and tp divides world."""
    if tp < 2 or tp > world or world % tp:
        raise ValueError(f"tp must divide the world size ({world}) and be at least 2")
    return [list(range(g * tp, (g + 1) * tp)) for g in range(world // tp)]


def tp_dp_rows(m: int, world: int, tp: int, rank: int):
    """Global Y rows [lo, hi) that ``rank`` owns in the tp x dp layout: its group's M slice
    (``m_slices(m, world/tp)``), then the fused reduce-scatter's band of that slice for the
    rank's position in the group (the slice must divide into tp equal bands)."""
    groups = tp_dp_groups(world, tp)
    g = rank // tp
    lo, hi = m_slices(m, len(groups))[g]
    if (hi - lo) % tp:
        raise ValueError("each group's M slice must divide into tp equal bands")
    per = (hi - lo) // tp
    pos = rank - g * tp
    return lo + pos * per, lo + (pos + 1) * per


class TpDpFusedFFN:
    """Two-level layout on one node: groups of ``tp`` GPUs each run the H-sharded FFN with
    the fused reduce-scatter (:class:`FusedTensorParallelFFN`, fp32 partials by default) on
    one M slice (``m_slices(M, world/tp)``); no communication between groups.  Each GPU
    sends (tp-1)/tp of its slice's partial Y instead of (P-1)/P of the whole batch's, so the
    NVLink bytes per GPU fall by about world/tp.  ``run`` returns this rank's rows
    ``local_rows()`` (global indices, ``tp_dp_rows``).

    Construction and :meth:`close` are collective over the whole world (every rank creates
    every group's communicator, in the same order)."""

    def __init__(self, x, w1, w2, *, tp=2, down_impl="basic", block_num=None, gelu="rational",
                 tile="cta128x256", partial="fp32"):
        import torch.distributed as dist

        world, rank = dist.get_world_size(), dist.get_rank()
        groups = tp_dp_groups(world, tp)
        self.groups = [dist.new_group(ranks) for ranks in groups]
        g = rank // tp
        k = x.shape[-1]
        m = x.numel() // k
        self.lo_rows, self.hi_rows = tp_dp_rows(m, world, tp, rank)
        lo, hi = m_slices(m, len(groups))[g]
        self.inner = FusedTensorParallelFFN(x.reshape(m, k)[lo:hi], w1, w2, group=self.groups[g],
                                            down_impl=down_impl, block_num=block_num, gelu=gelu, tile=tile,
                                            partial=partial)
        self.prepared = self.inner.prepared

    def launches_per_run(self):
        return 1

    def run(self):
        return self.inner.run()

    def local_rows(self):
        return list(range(self.lo_rows, self.hi_rows))

    def check(self):
        self.inner.check()

    def close(self):
        import torch.distributed as dist

        self.inner.close()
        dist.barrier()
