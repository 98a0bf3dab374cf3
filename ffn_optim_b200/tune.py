"""Implementation search: pick the fastest applicable, accurate implementation per case.

Mirrors the reference's outer tuning loop (performance/tune.py:6-31 and the evaluation
steps of performance/run.py:146-227): a serial, exhaustive walk over an explicit Cartesian
product of configurations.  Each configuration is prepared with no fallback (an
unavailable or inapplicable one is recorded as such, never replaced by another), checked
against an fp32 golden with the reference's acceptance rule, checked again on two repeated
invocations, then timed with unprofiled device events; the best is the passed
configuration with the smallest device median.  Every FFN call stays one kernel launch.

Beyond the reference's ``up_impl`` x ``down_impl`` axes the product may include this
build's ``tile`` (kernel variant) and ``schedule`` (static or claimed tile order) knobs.

Command line: ``python -m ffn_optim_b200.tune --workload cfg2_bf16`` prints one JSON
record per configuration and the best one.
"""
from __future__ import annotations

import itertools
import math

from .host.dispatch import DOWN_IMPLS, DependencyUnavailable, NotApplicable


def combinations(up, down, **axes):
    """Configurations of the Cartesian product, in order, duplicates removed (reference
    performance/tune.py:6-10).  ``up``/``down`` are the ``up_impl``/``down_impl`` search
    spaces; further keyword axes (e.g. ``tile=[None, 'pair256x256']``) are multiplied in."""
    spaces = [("up_impl", up), ("down_impl", down)] + list(axes.items())
    if any(not values for _, values in spaces):
        raise ValueError("Search spaces must be non-empty")
    names = [n for n, _ in spaces]
    values = [list(dict.fromkeys(v)) for _, v in spaces]
    return [dict(zip(names, combo)) for combo in itertools.product(*values)]


def search(configurations, evaluate, checkpoint=None):
    """Serial exhaustive search (reference performance/tune.py:13-31): ``evaluate(config)``
    returns a dict with ``status`` and ``device_median_us``; only ``status == 'passed'``
    with a finite positive median can win.  ``checkpoint(records, best)`` is called after
    every configuration and once more at the end."""
    records = []
    best = {"configuration": None, "device_median_us": None, "complete": False,
            "ranking_metric": "unprofiled_device_event_median_us", "scope": configurations}
    for configuration in configurations:
        row = dict(evaluate(configuration), configuration=configuration)
        records.append(row)
        value = row.get("device_median_us")
        if (row["status"] == "passed" and isinstance(value, (int, float)) and math.isfinite(value) and value > 0
                and (best["device_median_us"] is None or value < best["device_median_us"])):
            best.update(configuration=configuration, device_median_us=value)
        if checkpoint:
            checkpoint(records, best)
    best["complete"] = True
    if checkpoint:
        checkpoint(records, best)
    return records, best


def time_prepared(prepared, warmup=5, repeats=20):
    """Unprofiled device timing of ``prepared.run()`` (reference performance/collect.py):
    ``warmup`` untimed runs, then ``repeats`` runs each bracketed by CUDA events on the
    preparation stream; median and minimum in microseconds."""
    import torch

    for _ in range(warmup):
        prepared.run()
    prepared.check()
    pairs = []
    with torch.cuda.device(prepared.storage[0].device):
        # A device-side delay ahead of the timed launches keeps the stream's queue filled, so
        # each start event fires when the previous run ends rather than when the host gets
        # to the next launch (for short kernels the host launch would otherwise be timed).
        with torch.cuda.stream(prepared.stream):
            torch.cuda._sleep(100_000 * repeats)
        for _ in range(repeats):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(prepared.stream)
            prepared.run()
            end.record(prepared.stream)
            pairs.append((start, end))
        torch.cuda.synchronize()
    prepared.check()
    times = sorted(a.elapsed_time(b) * 1e3 for a, b in pairs)
    return {"device_median_us": times[len(times) // 2], "device_min_us": times[0], "repeats": repeats,
            "warmup": warmup}


def golden_rows(x, w1, w2, rows):
    """fp32 golden of the given rows (the reference's ``ffn_torch`` definition,
    validation/reference.py: exact-erf GELU, hidden kept in fp32) computed on the device
    in fp32 -- a check of the kernel's output, not a second implementation of the path."""
    import torch

    x2 = x.reshape(-1, x.shape[-1])[rows].float()
    hidden = torch.nn.functional.gelu(x2 @ w1.float().t())
    return hidden @ w2.float().t()


def evaluate_ffn(x, w1, w2, configuration, *, rows=256, warmup=5, repeats=20, block_num=None, seed=0):
    """One configuration, as performance/run.py:146-227 evaluates it: plan/prepare with no
    fallback, accuracy of the first and two repeated invocations on ``rows`` sampled rows
    against the fp32 golden (``compare``: mean relative error < 0.05), device timing.
    Returns a record with ``status`` in {'unavailable', 'not_applicable', 'compile_failed',
    'accuracy_failed', 'passed'}."""
    import torch

    from .api import KernelCompilationError, prepare_ffn
    from .metrics import compare

    row = {}
    config = {k: v for k, v in configuration.items() if v is not None}
    try:
        prepared = prepare_ffn(x, w1, w2, block_num=block_num, **config)
    except DependencyUnavailable as exc:
        return dict(row, status="unavailable", reason=str(exc), device_median_us=None)
    except NotApplicable as exc:
        return dict(row, status="not_applicable", reason=str(exc), device_median_us=None)
    except KernelCompilationError as exc:
        return dict(row, status="compile_failed", reason=str(exc), device_median_us=None)
    try:
        row["plan"] = {"variant": prepared.plan.kernel["variant"], "block_num": prepared.plan.block_num,
                       "schedule": prepared.plan.kernel.get("schedule")}
        m = prepared.plan.problem.m
        g = torch.Generator(device="cpu").manual_seed(seed)
        pick = torch.randperm(m, generator=g)[:min(rows, m)].sort().values.to(x.device)
        golden = golden_rows(x, w1, w2, pick)
        for attempt in range(3):  # the first invocation and two repeats
            out = prepared.run()
            prepared.check()
            got = out.reshape(-1, out.shape[-1])[pick].float()
            verdict = compare(got.cpu(), golden.cpu())
            if attempt == 0:
                row["accuracy"] = verdict
            if not verdict["passed"]:
                reason = "FP32 golden comparison failed" if attempt == 0 else "Repeated invocation failed"
                return dict(row, status="accuracy_failed", reason=reason, device_median_us=None)
        row.update(time_prepared(prepared, warmup, repeats))
        return dict(row, status="passed")
    finally:
        prepared.close()


def tune_ffn(x, w1, w2, *, up_candidates=("basic",), down_candidates=DOWN_IMPLS, tiles=(None,), schedules=(None,),
             warmup=5, repeats=20, rows=256, block_num=None, checkpoint=None):
    """Searches the product of the candidate lists for one (x, w1, w2); returns
    ``(records, best)`` as :func:`search`."""
    axes = {}
    if list(tiles) != [None]:
        axes["tile"] = list(tiles)
    if list(schedules) != [None]:
        axes["schedule"] = list(schedules)
    configurations = combinations(list(up_candidates), list(down_candidates), **axes)

    def evaluate(config):
        return evaluate_ffn(x, w1, w2, config, rows=rows, warmup=warmup, repeats=repeats, block_num=block_num)

    return search(configurations, evaluate, checkpoint)


def main(argv=None):
    import argparse
    import json

    import torch

    from . import cases as C

    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--workload", default="cfg2_bf16", help="case id of ffn_optim_b200/configs/cases.json")
    ap.add_argument("--up-candidates", nargs="+", default=["basic"])
    ap.add_argument("--down-candidates", nargs="+", default=list(DOWN_IMPLS))
    ap.add_argument("--tiles", nargs="+", default=None, help="kernel variants to search (default: automatic)")
    ap.add_argument("--schedules", nargs="+", default=None, choices=("static", "dynamic", "static_synced"))
    ap.add_argument("--block-num", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=20)
    args = ap.parse_args(argv)
    case = C.get_case(args.workload)
    x, w1, w2 = C.make_inputs(case, device="cuda")
    torch.cuda.synchronize()
    records, best = tune_ffn(x, w1, w2, up_candidates=args.up_candidates, down_candidates=args.down_candidates,
                             tiles=args.tiles or (None,), schedules=args.schedules or (None,),
                             warmup=args.warmup, repeats=args.repeats, block_num=args.block_num)
    for r in records:
        print(json.dumps({k: v for k, v in r.items() if k != "accuracy"} | {"case_id": args.workload}))
    print(json.dumps({"best": best["configuration"], "device_median_us": best["device_median_us"],
                      "case_id": args.workload}))
    return 0 if best["configuration"] is not None else 1


if __name__ == "__main__":
    raise SystemExit(main())
