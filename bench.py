"""Benchmark of the fused FFN hot path (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5_bf16] [--shard hf|h|m]

One step = one pass of the fused FFN over the workload's batch.  Default workload:
BASELINE configuration 5 (X[32,2048,8192], W1[28672,8192], W2[8192,28672], bf16), the
configuration the metric is quoted on at 1/2/4/8 GPUs.  Its inputs (1.0 GB X, 0.94 GB
weights) are larger than the 126 MB L2, so no flush is needed between steps.

Inputs are the case's seeded inputs (``ffn_optim_b200.cases``: PCG64 weights, X rows of the
golden fixture regenerated exactly, the other X rows drawn on the device), so every run
checks its own output rows against the reference's golden fixture (``tests/golden``) --
``parity`` in the line, at every N.

Keys: ``value`` = useful TFLOP/s (2*M*(K*H + H*N) per step, whole job) with inputs resident
in HBM.  N = 1: one fused kernel per step.  N > 1 (``--shard``, default ``hf``): H-sharded
tensor parallelism with the reduce-scatter fused into the kernel (partial tiles pushed over
NVLink as fp32); ``variants`` holds the same step timed with the M-sharded (no
communication), NCCL reduce-scatter, 24-bit-partial and input-dtype-partial variants,
and (N >= 4) the fused reduce-scatter inside pairs of GPUs with M split over the pairs.  ``e2e`` = the same
metric through the public API with X copied from pinned host memory and Y read back every
step (N = 1: ``PreparedFFN.run_host``; N > 1: ``RowShardedFFN.run_host`` on every rank, the
partitioning that moves each host byte over PCIe once).  ``roofline`` = the fused kernel
against the measured bf16 peak; ``cpu_baseline`` = the reference's own torch path
(``validation/reference.py::ffn_torch`` from the reference installed in ``baseline/_ref``;
the numpy port of it when that is absent) on a bounded row sample, with a parity check of
the GPU rows against it.  ``per_config`` (N = 1) times the other BASELINE configurations in
the same run, each with its roofline fraction and golden-fixture parity.  ``--impl
reference`` times the CPU reference alone (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused FFN useful TFLOP/s and µs/call at 1/2/4/8 B200; % of bf16 TC peak"
L2_BYTES = 128 << 20
GOLDEN = ROOT / "tests" / "golden"
REFERENCE_INSTALL = ROOT / "baseline" / "_ref"

# (workload, down_impl, weights) timed in the per_config block; cfg5 is the headline line.
PER_CONFIG = [("cfg1_fp16", "basic", "native"), ("cfg1_fp16", "streamk", "native"),
              ("cfg1_fp16", "full_load_a", "native"),
              ("cfg2_fp16", "streamk", "native"), ("cfg2_fp16", "full_load_a", "native"),
              ("cfg2_bf16", "streamk", "native"), ("cfg2_bf16", "full_load_a", "native"),
              ("cfg3_bf16", "streamk", "native"), ("cfg3_bf16", "streamk", "fp8"),
              ("cfg4_bf16", "basic", "native")]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg5_bf16")
    ap.add_argument("--shard", choices=("h", "hf", "m"), default="hf",
                    help="N>1: hf = H-sharded with the reduce-scatter fused into the kernel (NVLink peer stores, "
                         "fp32 partials), h = H-sharded + NCCL reduce-scatter, m = M-sharded")
    ap.add_argument("--chunks", type=int, default=4)
    ap.add_argument("--tile", default=None, help="force a kernel variant (see ffn_optim_b200._lib.TILE_VARIANTS)")
    ap.add_argument("--down-impl", choices=("basic", "streamk", "full_load_a"), default=None,
                    help="override the workload's down_impl")
    ap.add_argument("--weights", choices=("native", "fp8"), default="native",
                    help="fp8: e4m3 weights with per-row scales, widened on chip (decode tiles, M <= 64)")
    ap.add_argument("--schedule", choices=("static", "dynamic", "static_synced"), default=None,
                    help="data-parallel tile order (default: static_synced for CTA-pair tiles, static otherwise; "
                         "static_synced: static with each wave started after every owner started the previous one)")
    ap.add_argument("--raster-group", type=int, default=None,
                    help="N=1: tile rows per raster group (default: the planner's balanced choice)")
    ap.add_argument("--cpu-rows", type=int, default=1024)
    ap.add_argument("--flush", choices=("auto", "on", "off"), default="auto",
                    help="flush L2 between timed steps (auto: when the operands fit in 2x L2)")
    ap.add_argument("--e2e-chunks", type=int, default=8)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--no-variants", action="store_true", help="N>1: time only the --shard variant")
    ap.add_argument("--rows", type=int, default=None,
                    help="override M (the workload's K, H, N and weights; X drawn on the device; no golden "
                         "fixture, so no parity key): e.g. --workload cfg3_bf16 --rows 64 runs the swap64 decode tiles")
    return ap.parse_args()


def flops(p):
    return 2.0 * p.m * (p.k * p.h + p.h * p.n)


def unique_bytes(p, weight_bytes=2):
    """Algorithmic bytes of one call: X, W1, W2 and Y once each (hidden round trip excluded);
    fp8 weights count one byte per element plus their fp32 row scales."""
    w = (p.h * p.k + p.n * p.h) * weight_bytes + (4 * (p.h + p.n) if weight_bytes == 1 else 0)
    return 2 * (p.m * p.k + p.m * p.n) + w


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def traffic_for(workload, variant):
    """DRAM bytes per launch of the kernel variant that ran on this workload, from the
    committed ncu summary ("<workload>/<variant>" keys), if any."""
    f = ROOT / "profiles" / "traffic.json"
    if f.exists():
        d = json.loads(f.read_text())
        return d.get(f"{workload}/{variant}")
    return None


def kernel_name(variant):
    """The CUDA kernel a tile variant runs."""
    if variant and variant.startswith("hslice"):
        return "ffn_hslice_kernel"
    if variant and variant.startswith("rowblock"):
        return "ffn_rowblock_kernel"
    return "ffn_fused_kernel"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons around the timed region.

    Sampling starts before the timed region (nvidia-smi needs a moment to produce its first
    line); every sample carries nvidia-smi's timestamp and only samples inside
    [begin, end] of the timed region count -- or, when the region is shorter than the
    sampling period, the samples closest to it."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.02)
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def begin(self):
        self.window = [time.time(), None]

    def end(self):
        if self.window:
            self.window[1] = time.time()
        time.sleep(0.12)  # let the sample after the region arrive

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        from datetime import datetime

        samples = []
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                stamp = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                ts = time.mktime(stamp.timetuple()) + stamp.microsecond / 1e6
                samples.append((ts, float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        inside = samples
        if self.window and self.window[1] and samples:
            b, e = self.window
            inside = [x for x in samples if b - 0.05 <= x[0] <= e + 0.05]
            if not inside:  # region shorter than the sampling period: the nearest samples
                inside = sorted(samples, key=lambda x: min(abs(x[0] - b), abs(x[0] - e)))[:2]
        sm = [x[1] for x in inside]
        reasons = sorted({name for x in inside for name, val in zip(self.REASONS, x[4]) if val.lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": inside[0][2] if inside else None,
                "reasons": reasons, "samples": len(inside), "power_w_max": max(x[3] for x in inside) if inside else None}


# ------------------------------------------------------------------------------ inputs
def _tensor(bits, dtype, device):
    import numpy as np
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(dtype).to(device)


def case_inputs(case, device, world=1, rank=0, rows=None):
    """The case's seeded inputs on `device` and its golden fixture.

    Weights: the case's PCG64 streams (rank 0 draws them and broadcasts when world > 1).
    X: the whole seeded X when it is small; for large M, X drawn on the device (torch
    generator, seed 7: identical on every rank) with the fixture's rows regenerated exactly,
    since rows are independent and only those rows are checked."""
    import numpy as np
    import torch

    from ffn_optim_b200 import cases as C

    if rows is not None:  # the workload's weights with `rows` tokens; no fixture for this shape
        case = dict(case, shape=[rows, case["shape"][-1]], x_view="plain", noncontiguous=False)
    p = C.case_problem(case)
    dt = getattr(torch, p.dtype)
    fx = None if rows is not None else dict(np.load(GOLDEN / f"{case['case_id']}.npz"))
    if p.m <= 8192 and fx is not None:
        x, w1, w2 = C.make_inputs(case, device=device)
        return p, x, w1, w2, fx
    g = torch.Generator(device=device).manual_seed(7)
    x = torch.randn((p.m, p.k), generator=g, device=device, dtype=torch.float32).to(dt)
    if fx is not None:
        fixture_rows = torch.as_tensor(fx["rows"], device=device)
        x[fixture_rows] = _tensor(C.logical_x_rows(case, fx["rows"]), dt, device)
    if world == 1 or rank == 0:
        w1b, w2b = C.weights(case)
        w1, w2 = _tensor(w1b, dt, device), _tensor(w2b, dt, device)
    else:
        w1 = torch.empty((p.h, p.k), dtype=dt, device=device)
        w2 = torch.empty((p.n, p.h), dtype=dt, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.broadcast(w1, 0)
        dist.broadcast(w2, 0)
    return p, x.view(p.input_shape), w1, w2, fx


# ------------------------------------------------------------------------------ parity
def bits_to_f32(bits, dtype):
    import numpy as np

    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    if dtype == "bfloat16":
        return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def f32_to_bits(a, dtype):
    import numpy as np

    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == "float16":
        return a.astype(np.float16).view(np.uint16)
    u = a.view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def parity_vs_golden(got, fx, dtype, fp8=False):
    """Output rows (float32 values of the kernel's output dtype) against the reference's
    golden fixture: the reference criterion with the north-star max-abs bound against the
    exact-erf golden (``compare(strict=True)``), and two output ulps + 1e-3*max|golden| against
    the golden of the kernel's own arithmetic (rational GELU, staged hidden).  fp8 weights:
    relative RMS error < 0.05 against the golden (quantized weights, not the reference's
    arithmetic)."""
    import numpy as np
    import torch

    from ffn_optim_b200 import compare

    gold = bits_to_f32(fx["golden"], dtype)
    staged = bits_to_f32(fx["staged_rational"], dtype)
    r = compare(torch.from_numpy(got), torch.from_numpy(gold), strict=True)
    out = {"rows": int(got.shape[0]), "mean_rel": r["mean_rel"], "max_abs": r["max_abs"],
           "max_abs_ok": r["max_abs_ok"], "criterion": bool(r["passed"])}
    if fp8:
        rel_rms = float(np.sqrt(np.mean((got - gold) ** 2)) / np.sqrt(np.mean(gold ** 2)))
        out.update(rel_rms=rel_rms, passed=bool(rel_rms < 0.05), rule="fp8 weights: relative RMS < 0.05 vs golden")
        return out
    rel = 2.0 ** -6 if dtype == "bfloat16" else 2.0 ** -9
    excess = float((np.abs(got - staged) - (rel * np.abs(staged) + 1e-3 * np.abs(staged).max())).max())
    out.update(ulp_bound_excess=excess, passed=bool(r["passed"] and excess <= 0),
               rule="compare(strict=True) vs golden and <= 2 ulp + 1e-3*max vs staged rational golden")
    return out


def gather_rows(y_local, owned, rows, n, world):
    """The global output rows `rows` as float32 on rank 0: each rank fills the rows it owns
    (`owned`: global row -> local row of y_local), an all-reduce sums the disjoint parts."""
    import torch

    buf = torch.zeros((len(rows), n), dtype=torch.float32, device=y_local.device)
    y2 = y_local.reshape(-1, y_local.shape[-1])
    for i, r in enumerate(rows):
        j = owned(int(r))
        if j is not None:
            buf[i] = y2[j, :n].float()
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(buf)
    return buf.cpu().numpy()


# ------------------------------------------------------------------------------ CPU reference
def reference_ffn():
    """The reference's own torch golden path (validation/reference.py::ffn_torch) from the
    installed reference in baseline/_ref, or None when it is not installed."""
    if not (REFERENCE_INSTALL / "validation" / "reference.py").exists():
        return None
    sys.path.insert(0, str(REFERENCE_INSTALL))
    try:
        from validation.reference import ffn_torch
    except Exception:  # noqa: BLE001 - an unusable install falls back to the port
        return None
    finally:
        sys.path.remove(str(REFERENCE_INSTALL))
    return ffn_torch


def cpu_sample(p, xs, w1c, w2c, repeats=1):
    """Times the CPU baseline on the rows `xs` (CPU tensors of the input dtype): the
    reference's ffn_torch (kind 'reference'), else the numpy port of it (kind 'port').
    Returns (TFLOP/s, seconds, output float32 [rows, N], kind, threads)."""
    import torch

    ref = reference_ffn()
    best, out = None, None
    for _ in range(repeats):
        t0 = time.perf_counter()
        if ref is not None:
            with torch.no_grad():
                y = ref(xs, w1c, w2c)
        else:
            from oracle import ffn_oracle as O

            f = lambda t: t.float().numpy()  # noqa: E731
            y = O.ffn(f(xs), f(w1c), f(w2c), p.dtype)
        dt = time.perf_counter() - t0
        if best is None or dt < best:
            best, out = dt, y
    if ref is not None:
        out = out.float().numpy()
        kind, threads = "reference", torch.get_num_threads()
    else:
        out = bits_to_f32(out, p.dtype)
        kind, threads = "port", os.cpu_count()
    fl = 2.0 * xs.shape[0] * (p.k * p.h + p.h * p.n)
    return fl / best / 1e12, best, out, kind, threads


def run_reference(args):
    """--impl reference: the reference's CPU torch path on a row sample, rank 0 only."""
    import numpy as np
    import torch

    from ffn_optim_b200 import cases as C

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    case = C.get_case(args.workload)
    p = C.case_problem(case)
    dt = getattr(torch, p.dtype)
    rows = min(args.cpu_rows // 2 if p.m > 4096 else p.m, p.m)
    rng = np.random.Generator(np.random.PCG64(11))
    w1b, w2b = C.weights(case)
    xs = _tensor(C.logical_x_rows(case, np.sort(rng.choice(p.m, size=rows, replace=False))), dt, "cpu")
    w1c, w2c = _tensor(w1b, dt, "cpu"), _tensor(w2b, dt, "cpu")
    for _ in range(args.warmup):
        cpu_sample(p, xs, w1c, w2c)
    times = []
    kind = threads = None
    for _ in range(args.steps):
        _, sec, _, kind, threads = cpu_sample(p, xs, w1c, w2c)
        times.append(sec)
    total = sum(times)
    fl = 2.0 * rows * (p.k * p.h + p.h * p.n)
    value = fl * len(times) / total / 1e12
    what = "validation/reference.py::ffn_torch (installed reference, torch CPU)" if kind == "reference" else \
        "numpy port of validation/reference.py::ffn_torch (reference not installed)"
    sample = f"{rows} of {p.m} seeded rows of {args.workload} per step (rows are independent), full weights; {what}"
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / len(times) * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (bf16 inputs)",
            "data": "synthetic", "config": {"workload": args.workload, "rows_per_step": rows},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ timing
def timed(step, steps, scrub=None):
    """Device time (ms) of `steps` calls of `step` on the current stream: one event pair
    around all of them, or, with `scrub` (an L2-sized buffer), one pair per call with an L2
    flush between calls (flush not timed)."""
    import torch

    if scrub is None:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            step()
        e.record()
        e.synchronize()
        return s.elapsed_time(e)
    pairs = []
    for _ in range(steps):
        scrub.fill_(1.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step()
        e.record()
        pairs.append((s, e))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in pairs)


def sync_all(world):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(ms, dev, world):
    import torch

    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_runner(kind, x, w1, w2, down, args, world):
    """(runner, step, launches per step, parallelism label, owned-row map, output getter)."""
    from ffn_optim_b200 import prepare_ffn

    if world == 1:
        r = prepare_ffn(x, w1, w2, down_impl=down, tile=args.tile, schedule=args.schedule,
                        raster_group=args.raster_group,
                        weight_format=None if args.weights == "native" else args.weights)
        return r, r.run, 1, "single", (lambda g: g), r.run
    if kind in ("hf", "hf_fp24", "hf_input"):
        from ffn_optim_b200.sharded import FusedTensorParallelFFN

        partial = {"hf": "fp32", "hf_fp24": "fp24", "hf_input": "input"}[kind]
        r = FusedTensorParallelFFN(x, w1, w2, down_impl=down, partial=partial)
        lo = r.local_rows()[0]
        per = len(r.local_rows())
        owned = lambda g: g - lo if lo <= g < lo + per else None  # noqa: E731
        label = f"tp-h{world} (reduce-scatter fused in the kernel, NVLink peer stores, {partial} partials)"
        return r, r.run, 1, label, owned, r.run
    if kind == "hf_tp2":
        from ffn_optim_b200.sharded import TpDpFusedFFN

        r = TpDpFusedFFN(x, w1, w2, tp=2, down_impl=down)
        lo = r.lo_rows
        per = r.hi_rows - r.lo_rows
        owned = lambda g: g - lo if lo <= g < lo + per else None  # noqa: E731
        label = f"tp2 x dp{world // 2} (fused reduce-scatter inside each pair of GPUs, fp32 partials; M split over the pairs)"
        return r, r.run, 1, label, owned, r.run
    if kind == "h":
        from ffn_optim_b200.sharded import TensorParallelFFN

        r = TensorParallelFFN(x, w1, w2, chunks=args.chunks, down_impl=down, tile=args.tile)
        pos = {g: i for i, g in enumerate(r.local_rows())}
        return r, r.run, r.launches_per_run(), f"tp-h{world} (NCCL reduce-scatter, {r.launches_per_run()} M-chunks)", \
            pos.get, r.run
    from ffn_optim_b200.sharded import RowShardedFFN

    r = RowShardedFFN(x, w1, w2, down_impl=down, tile=args.tile, schedule=args.schedule)
    owned = lambda g: g - r.lo if r.lo <= g < r.hi else None  # noqa: E731
    return r, r.run, 1, f"m-shard{world}", owned, r.run


def close_runner(r):
    if hasattr(r, "close"):
        r.close()


# ------------------------------------------------------------------------------ per-config block
def per_config(dev, burst, hbm, warmup):
    """The other BASELINE configurations, timed in this run on one GPU with their parity
    against the golden fixture."""
    import numpy as np
    import torch

    from ffn_optim_b200 import NotApplicable, prepare_ffn
    from ffn_optim_b200 import cases as C

    out = []
    scrub = torch.empty(4 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    cache = {}
    for cid, down, weights in PER_CONFIG:
        case = C.get_case(cid)
        if cid not in cache:
            cache.clear()
            cache[cid] = case_inputs(case, dev)
        p, x, w1, w2, fx = cache[cid]
        entry = {"workload": cid, "down_impl": down, "weights": weights}
        try:
            r = prepare_ffn(x, w1, w2, down_impl=down, weight_format=None if weights == "native" else weights)
        except NotApplicable as exc:
            entry["not_applicable"] = str(exc)
            out.append(entry)
            continue
        ub = unique_bytes(p, 1 if weights == "fp8" else 2)
        flush = ub < 2 * L2_BYTES
        for _ in range(warmup + 2):
            r.run()
        r.check()
        y = r.run()
        got = y.reshape(-1, p.n)[torch.as_tensor(fx["rows"], device=dev)].float().cpu().numpy()
        r.check()
        roof_s = max(flops(p) / (burst * 1e12), ub / (hbm * 1e9))
        steps = int(min(200, max(10, 0.02 / roof_s)))  # at least ~20 ms of roofline time
        torch.cuda.synchronize()
        ms = timed(r.run, steps, scrub if flush else None)
        r.check()
        t = ms / steps * 1e-3
        roof_tc, roof_hbm = flops(p) / (burst * 1e12), ub / (hbm * 1e9)
        var = {v: k for k, v in _lib_variants().items()}.get(r.plan.kernel["variant"] + 1)
        entry.update(us_per_call=t * 1e6, tflops=flops(p) / t / 1e12, tbps=ub / t / 1e12,
                     bound="tensor" if roof_tc >= roof_hbm else "hbm", roofline_frac=max(roof_tc, roof_hbm) / t,
                     roofline_us=max(roof_tc, roof_hbm) * 1e6, variant=var, block_num=r.plan.block_num,
                     row_split=r.plan.kernel.get("row_split"), steps=steps,
                     l2="flushed between calls" if flush else "operands larger than 2x L2, no flush",
                     parity=parity_vs_golden(got, fx, p.dtype, fp8=weights == "fp8"))
        out.append(entry)
        r.close()
        del r, y
    cache.clear()
    del scrub
    torch.cuda.empty_cache()
    return out


def _lib_variants():
    from ffn_optim_b200 import _lib

    return _lib.TILE_VARIANTS


# ------------------------------------------------------------------------------ main
def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    from ffn_optim_b200 import cases as C

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    case = C.get_case(args.workload)
    p, x, w1, w2, fx = case_inputs(case, dev, world, rank, args.rows)
    down = args.down_impl or case.get("down_impl", "basic")
    fx_rows = [int(r) for r in fx["rows"]] if fx is not None else []
    burst, sustained, hbm, src = peaks()
    ub = unique_bytes(p, 1 if args.weights == "fp8" else 2)
    flush = args.flush == "on" or (args.flush == "auto" and ub < 2 * L2_BYTES)
    scrub = torch.empty(4 * L2_BYTES // 4, dtype=torch.float32, device=dev) if flush else None
    fl = flops(p)

    # ---- the primary variant: timed with clocks sampled
    primary = args.shard if world > 1 else "single"
    runner, step, launches, parallelism, owned, output = make_runner(primary, x, w1, w2, down, args, world)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    runner.check()
    y = output()
    parity = None
    if fx is not None:
        parity = parity_vs_golden(gather_rows(y, owned, fx_rows, p.n, world), fx, p.dtype,
                                  fp8=args.weights == "fp8")
    runner.check()
    sampler = ClockSampler(local)
    sampler.start()
    sync_all(world)
    sampler.begin()
    ms = timed(step, args.steps, scrub)
    sampler.end()
    sync_all(world)
    clocks = sampler.stop()
    runner.check()
    ms_max = max_over_ranks(ms, dev, world)
    value = fl * args.steps / (ms_max / 1e3) / 1e12
    ms_step = ms_max / args.steps
    if world > 1:
        every = [None] * world
        dist.all_gather_object(every, clocks)
        clocks = dict(every[0])
        clocks["sm_mhz_per_rank"] = [c.get("sm_mhz") for c in every]
        clocks["reasons_any_rank"] = sorted({r for c in every for r in c.get("reasons", [])})
    plan = (runner.prepared if world > 1 and hasattr(runner, "prepared")
            else runner.chunks[0].prepared if world > 1 else runner).plan
    variant = {v: k for k, v in _lib_variants().items()}.get(plan.kernel["variant"] + 1)
    per_launch_ms = ms_step / launches
    # The launch's own work: one rank's share of the FLOPs, its M rows of X/Y plus the weights
    # it streams (the bound is whichever roof is slower at the measured peaks).
    ub_launch = unique_bytes(p, 1 if args.weights == "fp8" else 2) / world / launches
    hbm_bound = ub_launch / (hbm * 1e9) > fl / world / launches / (burst * 1e12)
    if hbm_bound:
        achieved = ub_launch / (per_launch_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "peak_kind": f"{src} HBM copy (MEASURED_PEAKS.json)" if src == "measured" else "fallback HBM"}
    else:
        achieved = fl / world / launches / (per_launch_ms / 1e3) / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": burst, "unit": "TFLOP/s", "frac": achieved / burst,
                    "peak_kind": f"{src} burst bf16 (MEASURED_PEAKS.json)" if src == "measured" else "fallback burst bf16",
                    "frac_of_sustained": achieved / sustained}
    traffic = traffic_for(args.workload, variant) if world == 1 else None
    roofline.update(traffic=traffic,
                    traffic_source=("profiles/traffic.json (ncu dram__bytes_read.sum + dram__bytes_write.sum, one "
                                    f"launch of {args.workload} with {variant})") if traffic else None,
                    kernel=kernel_name(variant), variant=variant, per_launch_us=per_launch_ms * 1e3)

    # ---- N = 1: end to end through the public API, CPU baseline with its parity check
    e2e = cpu = None
    if world == 1 and not args.no_e2e:
        xh = x.cpu().pin_memory()
        yh = torch.empty(p.output_shape, dtype=x.dtype, pin_memory=True)
        for _ in range(2):
            runner.run_host(xh, yh, chunks=args.e2e_chunks)
        torch.cuda.synchronize()
        ms2 = timed(lambda: runner.run_host(xh, yh, chunks=args.e2e_chunks), args.steps)
        runner.check()
        e2e = {"value": fl * args.steps / (ms2 / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms2 / args.steps,
               "h2d_bytes_per_step": p.m * p.k * x.element_size(), "d2h_bytes_per_step": p.m * p.n * x.element_size(),
               "api": f"PreparedFFN.run_host(pinned X, pinned Y, chunks={args.e2e_chunks})",
               "gpu_launches": args.e2e_chunks * args.steps}
        del xh, yh
    if world == 1 and rank == 0 and not args.no_cpu and args.weights == "native":
        rows = np.sort(np.random.Generator(np.random.PCG64(5)).choice(p.m, size=min(args.cpu_rows, p.m),
                                                                       replace=False))
        sel = torch.as_tensor(rows, device=dev)
        xs = x.reshape(p.m, p.k)[sel].cpu()
        got = runner.run().reshape(p.m, p.n)[sel].float().cpu().numpy()
        runner.check()
        w1c, w2c = w1.cpu(), w2.cpu()
        tf, sec, ref_out, kind, threads = cpu_sample(p, xs, w1c, w2c)
        from ffn_optim_b200 import compare

        ref_t = torch.from_numpy(bits_to_f32(f32_to_bits(ref_out, p.dtype), p.dtype))
        chk = compare(torch.from_numpy(got), ref_t, strict=True)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": threads, "kind": kind,
               "sample": f"{len(rows)} of {p.m} rows of {args.workload} (full weights), {sec:.1f} s, "
                         + ("validation/reference.py::ffn_torch from baseline/_ref, torch CPU"
                            if kind == "reference" else "numpy port of validation/reference.py::ffn_torch"),
               "parity_of_gpu_rows": {"rows": len(rows), "mean_rel": chk["mean_rel"], "max_abs": chk["max_abs"],
                                      "passed": bool(chk["passed"]),
                                      "rule": "compare(strict=True): GPU rows vs the CPU reference's output"}}
        del w1c, w2c, xs

    # ---- N > 1: the other partitionings of the same step, each timed and checked
    variants = {}
    if world > 1 and not args.no_variants:
        close_runner(runner)
        del runner, step, output
        torch.cuda.empty_cache()
        kinds = ("m", "h", "hf_input", "hf_fp24") + (("hf_tp2",) if world >= 4 and world % 2 == 0 else ()) + ("hf",)
        for kind in [k for k in kinds if k != primary]:
            r, st, nl, label, own, outp = make_runner(kind, x, w1, w2, down, args, world)
            for _ in range(args.warmup):
                st()
            torch.cuda.synchronize()
            r.check()
            yv = outp()
            par = parity_vs_golden(gather_rows(yv, own, fx_rows, p.n, world), fx, p.dtype) if fx is not None else None
            r.check()
            sync_all(world)
            msv = timed(st, args.steps, scrub)
            sync_all(world)
            r.check()
            msv = max_over_ranks(msv, dev, world)
            variants[kind] = {"value": fl * args.steps / (msv / 1e3) / 1e12, "unit": "TFLOP/s",
                              "ms_per_step": msv / args.steps, "parallelism": label, "gpu_launches": nl * args.steps,
                              "parity": par}
            close_runner(r)
            del r, st, outp
            torch.cuda.empty_cache()
        runner = None

    # ---- N > 1 end to end: every rank streams its M-shard rows host -> device -> host
    if world > 1 and not args.no_e2e:
        from ffn_optim_b200.sharded import RowShardedFFN, m_slices

        ms_r = RowShardedFFN(x, w1, w2, down_impl=down)
        lo, hi = m_slices(p.m, world)[rank]
        xh = x.reshape(p.m, p.k)[lo:hi].cpu().pin_memory()
        yh = torch.empty((hi - lo, p.n), dtype=x.dtype, pin_memory=True)
        for _ in range(2):
            ms_r.run_host(xh, yh, chunks=args.e2e_chunks)
        sync_all(world)
        ms2 = timed(lambda: ms_r.run_host(xh, yh, chunks=args.e2e_chunks), args.steps)
        sync_all(world)
        ms_r.check()
        ms2 = max_over_ranks(ms2, dev, world)
        e2e = {"value": fl * args.steps / (ms2 / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms2 / args.steps,
               "h2d_bytes_per_step": p.m * p.k * x.element_size(), "d2h_bytes_per_step": p.m * p.n * x.element_size(),
               "api": f"RowShardedFFN.run_host on each rank (its M/{world} rows, pinned host X and Y, "
                      f"chunks={args.e2e_chunks}); bytes are whole-job",
               "gpu_launches": args.e2e_chunks * args.steps * world}
        ms_r.check()
        del ms_r, xh, yh

    configs = None
    if world == 1 and not args.no_per_config and args.workload == "cfg5_bf16" and args.rows is None:
        if runner is not None:
            close_runner(runner)
            runner = None
        del x, w1, w2
        torch.cuda.empty_cache()
        configs = per_config(dev, burst, hbm, args.warmup)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "us_per_call": ms_step * 1e3,
                "pct_bf16_peak": 100.0 * value / (burst * world), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16" if p.dtype == "bfloat16" else "f16",
                "data": "synthetic (seeded: PCG64 weights and fixture X rows of ffn_optim_b200.cases, other X rows "
                        "from a seeded device generator)",
                "config": {"workload": args.workload, "x": list(p.input_shape), "w1": [p.h, p.k], "w2": [p.n, p.h],
                           "down_impl": down, "parallelism": parallelism, "block_num": plan.block_num,
                           "kernel_variant": variant,
                           "schedule": {1: "static", 2: "dynamic", 3: "static_synced"}.get(plan.kernel.get("schedule")),
                           "weights": args.weights,
                           "l2": "L2 flushed between steps (512 MB write)" if flush else "inputs larger than L2, no flush"},
                "gpu_launches": launches * args.steps * world, "clocks": clocks, "roofline": roofline,
                "parity": parity, "e2e": e2e, "cpu_baseline": cpu}
        if variants:
            line["variants"] = variants
        if configs is not None:
            line["per_config"] = configs
        print(json.dumps(line), flush=True)
    if world > 1:
        if runner is not None:
            close_runner(runner)
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
