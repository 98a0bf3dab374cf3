"""Public API: ``ffn``, ``prepare_ffn`` and ``PreparedFFN`` (mirrors ops/api.py of the reference).

Same call signatures, argument meaning, return value (a view of a reused output buffer
that the next run overwrites) and error types.  Execution goes through the C ABI of the
sm_100a library; there is no CPU or torch fallback -- CPU tensors are rejected and a
missing library raises :class:`KernelCompilationError`.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from time import perf_counter

from . import _lib
from .host.dispatch import NotApplicable, Selection, kernel_provenance
from .host.inputs import pack_swiglu, prepare_storage, quantize_weights_fp8, validate_tensors
from .host.tiling import make_plan, problem_struct


class KernelCompilationError(RuntimeError):
    """The CUDA library could not be loaded or the kernel could not be set up
    (reference ops/api.py:9-14 wraps DSL compile failures the same way)."""


@dataclass
class PreparedFFN:
    """A prepared fused FFN that can be launched repeatedly (reference ops/api.py:17-45).

    ``storage`` is ``(x2d, w1, w2, hidden, out, workspace, counters, flags, status)`` on
    one CUDA device.  :meth:`run` launches one kernel on the preparation stream and returns
    ``out[:M, :N]`` viewed as ``(*x.shape[:-1], N)``; the view shares storage with the
    prepared buffer and the next run overwrites it.  Runs are asynchronous; :meth:`check`
    synchronises and raises if the kernel reported an error.
    """

    plan: object
    storage: tuple
    handle: object
    provenance: dict
    preparation: dict
    stream: object
    weight_scales: tuple = None  # fp8 weights: (W1 row scales [H], W2 row scales [N]); storage[1:3] hold the codes
    biases: tuple = None  # (bias1 [H] or None, bias2 [N] or None), 16-byte aligned device copies
    launch_overlap: bool = False  # see set_launch_overlap

    def _output_view(self):
        p = self.plan.problem
        return self.storage[4][:, :p.n].view(p.output_shape)

    def load_input(self, x):
        """Copies a new X (same shape/dtype; device tensor or pinned host tensor) into storage."""
        p = self.plan.problem
        if tuple(x.shape) != tuple(p.input_shape) or x.dtype != self.storage[0].dtype:
            raise ValueError("load_input: x must have the prepared shape and dtype")
        self.storage[0][:, :p.k].copy_(x.reshape(p.m, p.k), non_blocking=True)

    def run(self, x=None):
        """One FFN launch.  The returned view is overwritten by the next run."""
        import torch

        if self.handle is None:
            raise RuntimeError("PreparedFFN has been closed")
        with torch.cuda.device(self.storage[0].device):
            if torch.cuda.current_stream() != self.stream:
                raise RuntimeError("PreparedFFN must run on its preparation stream; concurrent reuse is unsupported")
            if x is not None:
                self.load_input(x)
            rc = _lib.load().ffn_b200_run(self.handle, ctypes.c_void_p(self.stream.cuda_stream))
            if rc != _lib.OK:
                raise RuntimeError(f"ffn_b200_run: {_lib.strerror(rc)}")
        return self._output_view()

    def capture_graph(self, runs=1):
        """Captures ``runs`` launches into a ``torch.cuda.CUDAGraph`` and returns it.

        ``graph.replay()`` on the preparation stream then re-runs them: each reads X from
        storage (``load_input`` or ``run(x)`` put it there) and writes the output view.  The
        launch epoch lives on the device, so replays, eager runs and other graphs of this
        FFN interleave freely; like runs, they must not overlap each other."""
        import torch

        if self.handle is None:
            raise RuntimeError("PreparedFFN has been closed")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.device(self.storage[0].device):
            side = torch.cuda.Stream()
            side.wait_stream(self.stream)
            with torch.cuda.graph(graph, stream=side):
                for _ in range(runs):
                    rc = _lib.load().ffn_b200_run(self.handle, ctypes.c_void_p(side.cuda_stream))
                    if rc != _lib.OK:
                        raise RuntimeError(f"ffn_b200_run (capture): {_lib.strerror(rc)}")
            self.stream.wait_stream(side)
        return graph

    def _chunk_handles(self, chunks):
        """Launch handles for M-chunks of this FFN (rows rounded to 128), sharing its storage:
        chunk c reads X rows [lo, hi), writes the same rows of hidden and Y, and has its own
        readiness counters; the fp32 Stream-K workspace is shared (chunks run in order on
        the preparation stream)."""
        import torch

        cached = getattr(self, "_chunks", None)
        if cached is not None and cached[0] == chunks:
            return cached[1]
        p = self.plan.problem
        rows = -(-p.m // chunks)
        rows = -(-rows // 128) * 128
        x2d, w1, w2, hidden, out, ws = self.storage[:6]
        lib = _lib.load()
        dev = x2d.device
        handles = []
        lo = 0
        while lo < p.m:
            hi = min(p.m, lo + rows)
            sub = self.plan.problem.__class__((hi - lo, p.k), hi - lo, p.k, p.h, p.n, p.dtype, p.layout)
            o = self.plan.kernel.get("overrides", {})
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            plan = make_plan(sub, self.plan.selection, self.plan.block_num, gelu=self.plan.gelu, sm_count=sms,
                             tile=o.get("tile"), raster_group=o.get("raster_group"), l2_policy=o.get("l2_policy"),
                             schedule=o.get("schedule"), weight_format=o.get("weight_format"))
            k = plan.kernel
            if self.plan.gelu == "swiglu" and k["swap_ab"] != self.plan.kernel["swap_ab"]:
                raise NotApplicable("run_host: a chunk's tiles need another SwiGLU row order of W1")
            if k["workspace_floats"] > ws.numel():
                ws = torch.empty(int(k["workspace_floats"]), dtype=torch.float32, device=dev)
            sync = torch.zeros(int(k["counter_words"]) + int(k["flag_words"]) + 4, dtype=torch.int32, device=dev)
            cnt, flg, st = sync[:k["counter_words"]], sync[k["counter_words"]:-4], sync[-4:]
            sc = self.weight_scales
            b1, b2 = self.biases or (None, None)
            bufs = _lib.Buffers(x2d[lo].data_ptr(), x2d.stride(0), w1.data_ptr(), w1.stride(0), w2.data_ptr(),
                                w2.stride(0), hidden[lo].data_ptr(), hidden.stride(0), out[lo].data_ptr(),
                                out.stride(0), ws.data_ptr(), cnt.data_ptr(), flg.data_ptr(), st.data_ptr(),
                                sc[0].data_ptr() if sc else None, sc[1].data_ptr() if sc else None,
                                b1.data_ptr() if b1 is not None else None, b2.data_ptr() if b2 is not None else None)
            prob = problem_struct(sub, self.plan.selection.down_impl, self.plan.gelu, plan.block_num, sms,
                                  o.get("tile"), o.get("raster_group"), o.get("l2_policy"), o.get("schedule"),
                                  o.get("weight_format"))
            h = ctypes.c_void_p()
            rc = lib.ffn_b200_prepare(ctypes.byref(prob), ctypes.byref(bufs), dev.index or 0, ctypes.byref(h))
            if rc != _lib.OK:
                raise _map_prepare_error(rc)
            if self.launch_overlap:
                lib.ffn_b200_set_launch_overlap(h, 1)
            handles.append((lo, hi, h, (ws, sync)))
            lo = hi
        self._chunks = (chunks, handles)
        self._chunk_streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        self._chunk_events = {}
        return handles

    def run_host(self, x_host, y_host, chunks=8):
        """FFN from host memory to host memory with the copies overlapped.

        ``x_host`` (``x.shape``) and ``y_host`` (``(*x.shape[:-1], N)``) are CPU tensors, pinned
        for asynchronous copies.  M is split into ``chunks`` row ranges; chunk c's host->device
        copy, fused kernel and device->host copy run on three streams so transfers overlap the
        other chunks' kernels.  Returns ``y_host``; like :meth:`run` it is asynchronous: the
        preparation stream waits for the last copy, so synchronising it (or :meth:`check`)
        completes the call.
        """
        import torch

        p = self.plan.problem
        if tuple(x_host.shape) != tuple(p.input_shape) or tuple(y_host.shape) != tuple(p.output_shape):
            raise ValueError("run_host: x_host / y_host must have the input / output shapes")
        if x_host.dtype != self.storage[0].dtype or y_host.dtype != self.storage[0].dtype:
            raise ValueError("run_host: host buffers must have the prepared dtype")
        handles = self._chunk_handles(chunks)
        h2d, d2h = self._chunk_streams
        lib = _lib.load()
        x2d, out = self.storage[0], self.storage[4]
        xs, ys = x_host.reshape(p.m, p.k), y_host.reshape(p.m, p.n)
        ev = self._chunk_events
        with torch.cuda.device(x2d.device):
            if torch.cuda.current_stream() != self.stream:
                raise RuntimeError("PreparedFFN must run on its preparation stream; concurrent reuse is unsupported")
            for lo, hi, h, _ in handles:
                key = lo
                done_k, done_out = ev.get(("k", key)), ev.get(("o", key))
                with torch.cuda.stream(h2d):
                    if done_k is not None:
                        h2d.wait_event(done_k)  # the previous kernel of this chunk has read X
                    x2d[lo:hi, :p.k].copy_(xs[lo:hi], non_blocking=True)
                    e_in = torch.cuda.Event()
                    e_in.record(h2d)
                self.stream.wait_event(e_in)
                if done_out is not None:
                    self.stream.wait_event(done_out)  # the previous copy-out of these Y rows finished
                rc = lib.ffn_b200_run(h, ctypes.c_void_p(self.stream.cuda_stream))
                if rc != _lib.OK:
                    raise RuntimeError(f"ffn_b200_run: {_lib.strerror(rc)}")
                e_k = torch.cuda.Event()
                e_k.record(self.stream)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(e_k)
                    ys[lo:hi].copy_(out[lo:hi, :p.n], non_blocking=True)
                    e_o = torch.cuda.Event()
                    e_o.record(d2h)
                ev[("k", key)], ev[("o", key)] = e_k, e_o
            for lo, _, _, _ in handles:
                self.stream.wait_event(ev[("o", lo)])
        return y_host

    def status(self):
        """Synchronises the stream and returns the kernel's status words [code, cta, aux, 0]."""
        self.stream.synchronize()
        return [int(v) for v in self.storage[8].tolist()]

    def check(self):
        """Raises RuntimeError if any launch since the last reset reported a device error
        (including the chunk launches of :meth:`run_host`)."""
        st = self.status()
        for _, _, _, (_, sync) in (getattr(self, "_chunks", None) or (0, []))[1]:
            cst = [int(v) for v in sync[-4:].tolist()]
            if cst[0] != 0:
                st = cst
                break
        if st[0] != 0:
            self.reset()
            msg = _lib.KERNEL_ERRORS.get(st[0], f"error {st[0]}")
            raise RuntimeError(f"fused FFN kernel failed: {msg} (cta {st[1]}, aux {st[2]})")
        return True

    def reset(self):
        """Clears counters, flags and status and restarts the launch epoch."""
        rc = _lib.load().ffn_b200_reset(self.handle, ctypes.c_void_p(self.stream.cuda_stream))
        if rc != _lib.OK:
            raise RuntimeError(f"ffn_b200_reset: {_lib.strerror(rc)}")

    def set_wait_limit(self, seconds: float):
        """Upper bound of every in-kernel wait; on expiry the kernel reports an error."""
        rc = _lib.load().ffn_b200_set_wait_limit(self.handle, int(seconds * 1e9))
        if rc != _lib.OK:
            raise ValueError(f"set_wait_limit: {_lib.strerror(rc)}")

    def set_launch_overlap(self, enable: bool = True):
        """Overlapped launches (programmatic dependent launch): each later ``run()`` sets up
        while the stream's previous kernel finishes and touches global memory only after
        that kernel completed, so results and ordering are those of serial launches; saves
        the launch gap of back-to-back calls.  Off by default."""
        handles = [self.handle] + [h for _, _, h, _ in (getattr(self, "_chunks", None) or (0, []))[1]]
        for h in handles:
            rc = _lib.load().ffn_b200_set_launch_overlap(h, 1 if enable else 0)
            if rc != _lib.OK:
                raise ValueError(f"set_launch_overlap: {_lib.strerror(rc)}")
        self.launch_overlap = bool(enable)

    def set_fault_injection(self, mode: int):
        """Test hook (1 = readiness waits can never be satisfied); see ffn_b200_set_fault_injection."""
        rc = _lib.load().ffn_b200_set_fault_injection(self.handle, int(mode))
        if rc != _lib.OK:
            raise ValueError(f"set_fault_injection: {_lib.strerror(rc)}")

    def trace(self):
        """Runs once with per-CTA %globaltimer stamps and returns a dict of phase times (us)
        relative to the earliest setup stamp: per-slot min/median/max over CTAs, and under
        "smid" the SM each CTA ran on (index = CTA)."""
        import torch

        grid = self.plan.block_num
        stamps = torch.zeros((grid, 16), dtype=torch.int64, device=self.storage[0].device)
        lib = _lib.load()
        if lib.ffn_b200_set_trace(self.handle, stamps.data_ptr()) != _lib.OK:
            raise RuntimeError("ffn_b200_set_trace failed")
        try:
            self.run()
            self.check()
        finally:
            lib.ffn_b200_set_trace(self.handle, None)
        t = stamps.cpu()
        t0 = int(t[:, 0][t[:, 0] > 0].min())
        names = {0: "start", 1: "first_load", 2: "down_ready", 3: "last_load", 4: "last_mma", 5: "up_stored",
                 6: "first_down", 7: "end", 9: "aux1", 10: "aux2", 11: "aux3", 12: "aux4", 13: "aux5", 14: "aux6",
                 15: "aux7"}
        out = {}
        for i, name in names.items():
            col = t[:, i][t[:, i] > 0].double()
            if col.numel():
                rel = (col - t0) / 1e3
                out[name] = {"min": float(rel.min()), "median": float(rel.median()), "max": float(rel.max()),
                             "ctas": int(col.numel())}
        out["smid"] = [int(v) for v in t[:, 8]]
        return out

    def set_owner_map(self, owners):
        """Work-list index of each CTA (CTA pair for pair tiles): a permutation of
        0..C-1, or None for launch order.  Only the tile-to-SM placement changes; every
        tile is still computed once by the same arithmetic."""
        import torch

        lib = _lib.load()
        if owners is None:
            self._owner_map = None
            rc = lib.ffn_b200_set_owner_map(self.handle, None)
        else:
            n = self.plan.block_num // (2 if self.plan.kernel["cta_pair"] else 1)
            owners = [int(v) for v in owners]
            if sorted(owners) != list(range(n)):
                raise ValueError(f"owner map must be a permutation of 0..{n - 1}")
            self._owner_map = torch.tensor(owners, dtype=torch.int32, device=self.storage[0].device)
            rc = lib.ffn_b200_set_owner_map(self.handle, self._owner_map.data_ptr())
        if rc != _lib.OK:
            raise RuntimeError(f"ffn_b200_set_owner_map: {_lib.strerror(rc)}")

    def owner_map(self):
        """The work-list index of each CTA (pair) in use, or None for launch order."""
        lib = _lib.load()
        cap = 1024
        buf = (ctypes.c_int32 * cap)()
        count = ctypes.c_int32(0)
        rc = lib.ffn_b200_get_owner_map(self.handle, buf, cap, ctypes.byref(count))
        if rc != _lib.OK:
            raise RuntimeError(f"ffn_b200_get_owner_map: {_lib.strerror(rc)}")
        return [int(v) for v in buf[:count.value]] if count.value else None

    def close(self):
        if self.handle is not None:
            _lib.load().ffn_b200_destroy(self.handle)
            self.handle = None
        for _, _, h, _ in (getattr(self, "_chunks", None) or (0, []))[1]:
            _lib.load().ffn_b200_destroy(h)
        self._chunks = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def _map_prepare_error(rc):
    msg = _lib.strerror(rc)
    if rc in (_lib.ERR_INVALID, _lib.ERR_ALIGNMENT, _lib.ERR_TOO_LARGE):
        return ValueError(f"prepare_ffn: {msg}")
    if rc == _lib.ERR_DEVICE:
        return RuntimeError(f"prepare_ffn: {msg}")
    return KernelCompilationError(f"prepare_ffn: {msg}")


def _prepared_bias(bias, features, x, name):
    """A bias vector as a contiguous, 16-byte aligned device tensor of x's dtype, or None."""
    import torch

    if bias is None:
        return None
    if not isinstance(bias, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor or None")
    if bias.dtype != x.dtype or bias.device != x.device or tuple(bias.shape) != (features,):
        raise ValueError(f"{name} must be a [{features}] tensor of the input's dtype on its device")
    if bias.requires_grad:
        raise ValueError(f"{name} must not require grad")
    if bias.is_contiguous() and bias.data_ptr() % 16 == 0:
        return bias
    out = torch.empty(features + 8, dtype=bias.dtype, device=bias.device)[:features]
    out.copy_(bias)
    return out


def prepare_ffn(x, weight1, weight2, *, up_impl="basic", down_impl="basic", block_num=None,
                layout="linear", gelu="rational", tile=None, raster_group=None, l2_policy=None, schedule=None,
                weight_format=None, activation="gelu", bias1=None, bias2=None):
    """Validates, plans and prepares storage and the launch handle without launching the FFN
    (reference ops/api.py:48-89).

    ``block_num`` is the persistent CTA count, at most the device's SM count (default: all
    SMs).  ``gelu`` selects the epilogue GELU: 'rational' (the reference kernel's clipped
    rational erf) or 'erf' (CUDA ``erff``).  ``tile`` forces a kernel variant (see
    ``make_plan``); None chooses automatically; ``raster_group``, ``l2_policy`` and
    ``schedule`` are tuning overrides passed to ``make_plan``.  ``weight_format='fp8'``
    (decode, M <= 64) quantizes W1 and W2 once to e4m3 codes with per-row fp32 scales
    (``quantize_weights_fp8``) and runs the tiles that widen them on chip: half the weight
    bytes, a weight-quantization error on top of the reference arithmetic.  Storage copies
    are device work timed separately as ``preparation['auxiliary_device_interval_ms']``.

    Beyond the reference's V1: ``layout='canonical'`` takes W1 as [K, H] and W2 as [H, N]
    (``Y = GELU(X W1) W2``), copied once into Linear storage; ``activation='silu'`` replaces
    the GELU by SiLU;
    ``activation='swiglu'`` takes ``weight1 = [W_gate; W_up]`` ([2H, K]) and computes
    ``hidden = SiLU(x W_gate^T) * (x W_up^T)``; ``bias1`` [H] / ``bias2`` [N] (input dtype) are
    added to the fp32 sums before the activation / before the final rounding (``bias1`` not
    with SwiGLU).
    """
    import torch

    if activation not in ("gelu", "silu", "swiglu"):
        raise ValueError("activation must be 'gelu', 'silu' or 'swiglu'")
    if gelu not in ("rational", "erf"):
        raise ValueError("gelu must be 'rational' or 'erf'")
    glu = activation == "swiglu"
    canonical = layout == "canonical"
    if canonical:
        # Canonical weights (W1 [K, H], W2 [H, N], X @ W1 without a transpose) are the same
        # weights stored transposed: validated and planned as their Linear views, then copied
        # once into Linear storage with the other preparation copies.
        if glu:
            raise ValueError("activation='swiglu' takes Linear weights (gate and up as row halves of weight1)")
        if not all(isinstance(w, torch.Tensor) and w.dim() == 2 for w in (weight1, weight2)):
            raise ValueError("layout='canonical' takes 2-D weight1 [K, H] and weight2 [H, N]")
        weight1, weight2, layout = weight1.t(), weight2.t(), "linear"
    if glu:
        # W1 = [gate rows; up rows], [2H, K]; validated as the gate half against W2 [N, H]
        if not isinstance(weight1, torch.Tensor) or weight1.dim() != 2 or isinstance(weight2, torch.Tensor) and (
                weight2.dim() != 2 or weight1.shape[0] != 2 * weight2.shape[1]):
            raise ValueError("activation='swiglu' takes weight1 = [gate; up] of shape [2H, K] and weight2 [N, H]")
        if bias1 is not None:
            raise ValueError("bias1 is not supported with activation='swiglu'")
        p = validate_tensors(x, weight1[:weight2.shape[1]], weight2, layout=layout, require_cuda=True)
    else:
        p = validate_tensors(x, weight1, weight2, layout=layout, require_cuda=True)
    act = activation if activation != "gelu" else gelu
    b1 = _prepared_bias(bias1, p.h, x, "bias1")
    b2 = _prepared_bias(bias2, p.n, x, "bias2")
    selection = Selection(up_impl, down_impl)
    try:
        lib = _lib.load()
    except (OSError, RuntimeError) as exc:
        raise KernelCompilationError(f"{type(exc).__name__}: {exc}") from exc
    props = torch.cuda.get_device_properties(x.device)
    plan = make_plan(p, selection, block_num, gelu=act, sm_count=props.multi_processor_count, tile=tile,
                     raster_group=raster_group, l2_policy=l2_policy, schedule=schedule, weight_format=weight_format)
    if (props.major, props.minor) != (10, 0):
        raise RuntimeError("This implementation targets B200 (sm_100) only")
    if plan.block_num > props.multi_processor_count:
        raise ValueError("Persistent grid requires block_num <= SM count")
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        scales = None
        if canonical:
            weight1, weight2 = weight1.contiguous(), weight2.contiguous()
        if glu:  # the kernel's gate/up row order
            weight1 = pack_swiglu(weight1, p.h, plan.kernel["swap_ab"])
        if weight_format == "fp8":
            q1, s1 = quantize_weights_fp8(weight1)
            q2, s2 = quantize_weights_fp8(weight2)
            weight1, weight2, scales = q1[:, :p.k], q2[:, :p.h], (s1, s2)
        storage = prepare_storage(x, weight1, weight2, plan)
        end.record()
        end.synchronize()
        auxiliary_ms = start.elapsed_time(end)
        x2d, w1, w2, hidden, out, ws, counters, flags, status = storage
        bufs = _lib.Buffers(x2d.data_ptr(), x2d.stride(0), w1.data_ptr(), w1.stride(0), w2.data_ptr(), w2.stride(0),
                            hidden.data_ptr(), hidden.stride(0), out.data_ptr(), out.stride(0), ws.data_ptr(),
                            counters.data_ptr(), flags.data_ptr(), status.data_ptr(),
                            scales[0].data_ptr() if scales else None, scales[1].data_ptr() if scales else None,
                            b1.data_ptr() if b1 is not None else None, b2.data_ptr() if b2 is not None else None)
        prob = problem_struct(p, down_impl, act, plan.block_num, props.multi_processor_count, tile, raster_group,
                              l2_policy, schedule, weight_format)
        handle = ctypes.c_void_p()
        before = perf_counter()
        rc = lib.ffn_b200_prepare(ctypes.byref(prob), ctypes.byref(bufs), x.device.index or 0, ctypes.byref(handle))
        if rc != _lib.OK:
            raise _map_prepare_error(rc)
        preparation = {"auxiliary_device_interval_ms": auxiliary_ms,
                       "compile_wall_ms": (perf_counter() - before) * 1000}
    provenance = kernel_provenance(down_impl)
    provenance["plan"] = plan.kernel
    return PreparedFFN(plan, storage, handle, provenance, preparation, stream, scales, (b1, b2))


def ffn(x, weight1, weight2, **configuration):
    """Y = GELU(X @ weight1.T) @ weight2.T; no bias, no autograd (reference ops/api.py:92-94)."""
    return prepare_ffn(x, weight1, weight2, **configuration).run()
