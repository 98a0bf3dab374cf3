"""Accuracy criterion (reference validation/test_ffn.py:6-21, extended).

``compare`` keeps the reference's result dict and pass rule -- shapes and dtypes equal,
both finite, mean(|a-b| / (|b| + 1e-3)) < 0.05 -- and adds the north-star bound
max|a-b| <= 2e-2 * max|b| as ``max_abs_ok``; ``strict=True`` requires both.
"""
from __future__ import annotations

MEAN_REL_LIMIT = 0.05
MAX_ABS_FRACTION = 2e-2


def compare(output, golden, *, strict=False):
    import torch

    result = {"passed": False, "shape_ok": tuple(output.shape) == tuple(golden.shape),
              "dtype_ok": output.dtype == golden.dtype, "finite": False,
              "max_abs": None, "rms": None, "mean_rel": None, "max_abs_ok": None}
    if not result["shape_ok"] or not result["dtype_ok"]:
        return result
    a, b = output.detach().float().cpu(), golden.detach().float().cpu()
    result["finite"] = bool(torch.isfinite(a).all() and torch.isfinite(b).all())
    if not result["finite"] or not a.numel():
        return result
    d = (a - b).abs()
    result.update(max_abs=d.max().item(), rms=d.square().mean().sqrt().item(),
                  mean_rel=(d / (b.abs() + 1e-3)).mean().item())
    result["max_abs_ok"] = result["max_abs"] <= MAX_ABS_FRACTION * b.abs().max().item()
    result["passed"] = result["mean_rel"] < MEAN_REL_LIMIT and (result["max_abs_ok"] or not strict)
    return result
