"""Benchmark of the fused FFN hot path (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5_bf16] [--shard h|m]

One step = one pass of the fused FFN over the workload's synthetic batch (for N > 1 the
H-sharded tensor-parallel step: per-rank fused kernels over M-chunks + NCCL reduce-scatter
of the partial Y).  Default workload: BASELINE configuration 5 (X[32,2048,8192],
W1[28672,8192], W2[8192,28672], bf16), the configuration the metric is quoted on at
1/2/4/8 GPUs.  Inputs (1.0 GB X, 0.94 GB weights) are larger than the 126 MB L2, so no
flush is needed between steps.

Keys: ``value`` = useful TFLOP/s (2*M*(K*H + H*N) per step, whole job) with inputs resident
in HBM; ``e2e`` = the same through the public API with X copied from pinned host memory
and Y read back every step; ``roofline`` = the fused kernel against the measured bf16 peak;
``cpu_baseline`` = the CPU oracle (numpy port of the reference's torch path) on a bounded
row sample.  ``--impl reference`` times that CPU path alone (rank 0 only).
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg5_bf16")
    ap.add_argument("--shard", choices=("h", "hf", "m"), default="m",
                    help="N>1: h = H-sharded + NCCL reduce-scatter, hf = H-sharded with the reduce-scatter "
                         "fused into the kernel (NVLink peer stores), m = M-sharded")
    ap.add_argument("--chunks", type=int, default=4)
    ap.add_argument("--tile", default=None, help="force a kernel variant (see ffn_optim_b200._lib.TILE_VARIANTS)")
    ap.add_argument("--down-impl", choices=("basic", "streamk", "full_load_a"), default=None,
                    help="override the workload's down_impl")
    ap.add_argument("--weights", choices=("native", "fp8"), default="native",
                    help="fp8: e4m3 weights with per-row scales, widened on chip (decode tiles, M <= 64)")
    ap.add_argument("--schedule", choices=("static", "dynamic"), default=None,
                    help="data-parallel tile order (default: dynamic for CTA-pair tiles, static otherwise)")
    ap.add_argument("--cpu-rows", type=int, default=1024)
    ap.add_argument("--flush", choices=("auto", "on", "off"), default="auto",
                    help="flush L2 between timed steps (auto: when the operands fit in 2x L2)")
    ap.add_argument("--e2e-chunks", type=int, default=8)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    return ap.parse_args()


def flops(p):
    return 2.0 * p.m * (p.k * p.h + p.h * p.n)


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def traffic_for(workload):
    """DRAM bytes per launch of the fused kernel from the committed ncu summary, if any."""
    f = ROOT / "profiles" / "traffic.json"
    if f.exists():
        d = json.loads(f.read_text())
        if workload in d:
            return d[workload]
    return None


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
                ts = time.mktime(datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timetuple()) + \
                    datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").microsecond / 1e6
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


def device_inputs(case, device, seed=7):
    """Synthetic inputs of the workload's shapes and distributions, generated on the GPU."""
    import torch

    from ffn_optim_b200 import cases as C

    p = C.case_problem(case)
    dt = getattr(torch, p.dtype)
    g = torch.Generator(device=device).manual_seed(seed)
    normal = case.get("distribution", "normal_fanin") == "normal_fanin"
    if normal:
        x = torch.randn(p.input_shape, generator=g, device=device, dtype=torch.float32).to(dt)
        w1 = (torch.randn((p.h, p.k), generator=g, device=device) * p.k ** -0.5).to(dt)
        w2 = (torch.randn((p.n, p.h), generator=g, device=device) * p.h ** -0.5).to(dt)
    else:
        x = (torch.rand(p.input_shape, generator=g, device=device) * 4 - 2).to(dt)
        w1 = (torch.randn((p.h, p.k), generator=g, device=device) * 0.05).to(dt)
        w2 = (torch.randn((p.n, p.h), generator=g, device=device) * 0.05).to(dt)
    return p, x, w1, w2


def cpu_oracle_sample(p, x_rows_bits, w1_bits, w2_bits, repeats=1):
    """Times the CPU oracle (numpy port of the reference's ffn_torch, including its per-call
    weight conversion to fp32) on a row sample; returns (TFLOP/s, seconds per call)."""
    from oracle import ffn_oracle as O

    rows = x_rows_bits.shape[0]
    best = None
    for _ in range(repeats):
        t0 = time.perf_counter()
        O.ffn(O.from_bits(x_rows_bits, p.dtype), O.from_bits(w1_bits, p.dtype), O.from_bits(w2_bits, p.dtype),
              p.dtype)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    fl = 2.0 * rows * (p.k * p.h + p.h * p.n)
    return fl / best / 1e12, best


def _lib_variants():
    from ffn_optim_b200 import _lib

    return _lib.TILE_VARIANTS


def to_bits(t):
    import numpy as np
    import torch

    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def run_reference(args):
    """--impl reference: the CPU oracle of the reference's torch path, rank 0 only."""
    import numpy as np

    from ffn_optim_b200 import cases as C

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    case = C.get_case(args.workload)
    p = C.case_problem(case)
    rows = min(args.cpu_rows // 2 if p.m > 4096 else p.m, p.m)
    rng = np.random.Generator(np.random.PCG64(11))
    def bf(shape, scale):
        from oracle import ffn_oracle as O
        return O.to_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale), p.dtype)
    xb = bf((rows, p.k), 1.0)
    w1b = bf((p.h, p.k), p.k ** -0.5)
    w2b = bf((p.n, p.h), p.h ** -0.5)
    cores = os.cpu_count()
    for _ in range(args.warmup):
        cpu_oracle_sample(p, xb, w1b, w2b)
    times = []
    for _ in range(args.steps):
        _, dt = cpu_oracle_sample(p, xb, w1b, w2b)
        times.append(dt)
    total = sum(times)
    fl = 2.0 * rows * (p.k * p.h + p.h * p.n)
    value = fl * len(times) / total / 1e12
    sample = f"{rows} of {p.m} rows of {args.workload} per step (rows are independent), full weights"
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / len(times) * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (bf16 inputs)",
            "data": "synthetic", "config": {"workload": args.workload, "rows_per_step": rows},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from ffn_optim_b200 import cases as C
    from ffn_optim_b200 import prepare_ffn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    case = C.get_case(args.workload)
    p, x, w1, w2 = device_inputs(case, dev)
    down = args.down_impl or case.get("down_impl", "basic")

    if world == 1:
        runner = prepare_ffn(x, w1, w2, down_impl=down, tile=args.tile, schedule=args.schedule,
                             weight_format=None if args.weights == "native" else args.weights)
        launches = 1
        kernel_runs = lambda: runner.run()  # noqa: E731
        check = runner.check
        parallelism = "single"
    elif args.shard == "hf":
        from ffn_optim_b200.sharded import FusedTensorParallelFFN

        runner = FusedTensorParallelFFN(x, w1, w2, down_impl=down)
        launches = 1
        kernel_runs = runner.run
        check = runner.check
        parallelism = f"tp-h{world} (reduce-scatter fused in the kernel, NVLink peer stores)"
    elif args.shard == "h":
        from ffn_optim_b200.sharded import TensorParallelFFN

        runner = TensorParallelFFN(x, w1, w2, chunks=args.chunks, down_impl=down, tile=args.tile)
        launches = runner.launches_per_run()
        kernel_runs = runner.run
        check = runner.check
        parallelism = f"tp-h{world} (reduce-scatter, {launches} M-chunks)"
    else:
        from ffn_optim_b200.sharded import RowShardedFFN

        runner = RowShardedFFN(x, w1, w2, down_impl=down, tile=args.tile, schedule=args.schedule)
        launches = 1
        kernel_runs = runner.run
        check = runner.check
        parallelism = f"m-shard{world}"
    del w1, w2

    for _ in range(args.warmup):
        kernel_runs()
    torch.cuda.synchronize()
    check()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    unique_bytes = 2 * (p.m * p.k + p.h * p.k + p.n * p.h + p.m * p.n)
    flush = args.flush == "on" or (args.flush == "auto" and unique_bytes < 2 * L2_BYTES)
    scrub = torch.empty(4 * L2_BYTES // 4, dtype=torch.float32, device=dev) if flush else None
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.begin()
    if flush:
        # Each step timed alone; an L2-sized write between steps evicts the operands.
        ms = 0.0
        pairs = []
        for _ in range(args.steps):
            scrub.fill_(1.0)
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            kernel_runs()
            e0.record()
            pairs.append((s0, e0))
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in pairs)
    else:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            kernel_runs()
        end.record()
        end.synchronize()
        ms = start.elapsed_time(end)
    sampler.end()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    check()
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    fl = flops(p)
    value = fl * args.steps / (ms_max / 1e3) / 1e12
    ms_step = ms_max / args.steps

    # End to end through the public API: pinned host X in, Y out, every step.
    e2e = None
    if world == 1 and not args.no_e2e:
        xh = x.cpu().pin_memory()
        yh = torch.empty(p.output_shape, dtype=x.dtype, pin_memory=True)
        chunks = args.e2e_chunks
        for _ in range(2):
            runner.run_host(xh, yh, chunks=chunks)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            runner.run_host(xh, yh, chunks=chunks)
        e2.record()
        e2.synchronize()
        ms2 = s2.elapsed_time(e2)
        check()
        e2e = {"value": fl * args.steps / (ms2 / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms2 / args.steps,
               "h2d_bytes_per_step": p.m * p.k * x.element_size(), "d2h_bytes_per_step": p.m * p.n * x.element_size(),
               "api": f"PreparedFFN.run_host(pinned X, pinned Y, chunks={chunks})", "gpu_launches": chunks * args.steps}

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu and args.weights == "native":
        rows = min(args.cpu_rows, p.m)
        xb = to_bits(x.reshape(p.m, p.k)[:rows])
        w1b = to_bits(runner.storage[1][:, :p.k])
        w2b = to_bits(runner.storage[2][:, :p.h])
        tf, sec = cpu_oracle_sample(p, xb, w1b, w2b)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{rows} of {p.m} rows of {args.workload} (full weights), {sec:.1f} s, numpy float32 BLAS"}

    first = runner if world == 1 else (runner.chunks[0].prepared if hasattr(runner, "chunks") else runner.prepared)
    block_num = first.plan.block_num
    variant = {v: k for k, v in _lib_variants().items()}.get(first.plan.kernel["variant"] + 1)
    burst, sustained, hbm, src = peaks()
    per_launch_ms = ms_step / launches
    flops_launch = fl / world / launches
    achieved = flops_launch / (per_launch_ms / 1e3) / 1e12
    traffic = traffic_for(args.workload) if world == 1 else None
    roofline = {"bound": "tensor", "achieved": achieved, "peak": burst, "unit": "TFLOP/s", "frac": achieved / burst,
                "traffic": traffic, "peak_kind": f"{src} burst bf16", "frac_of_sustained": achieved / sustained,
                "kernel": "ffn_fused_kernel", "per_launch_us": per_launch_ms * 1e3}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "us_per_call": ms_step * 1e3,
                "pct_bf16_peak": 100.0 * value / (burst * world), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16" if p.dtype == "bfloat16" else "f16", "data": "synthetic",
                "config": {"workload": args.workload, "x": list(p.input_shape), "w1": [p.h, p.k], "w2": [p.n, p.h],
                           "down_impl": down, "parallelism": parallelism,
                           "block_num": block_num, "kernel_variant": variant,
                           "schedule": {1: "static", 2: "dynamic"}.get(first.plan.kernel.get("schedule")),
                           "weights": args.weights,
                           "l2": "L2 flushed between steps (512 MB write)" if flush else "inputs larger than L2, no flush"},
                "gpu_launches": launches * args.steps, "clocks": clocks, "roofline": roofline,
                "e2e": e2e, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
