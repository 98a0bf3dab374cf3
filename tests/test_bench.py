"""The parts of ``bench.py``'s contract that need no GPU: the work counts its throughput and
roofline figures divide by (FLOPs = 2*M*(K*H + H*N), unique bytes = X, W1, W2 and Y once),
the golden-fixture parity rule its ``parity`` keys apply, and the reference arm's JSON line
(``--impl reference``: the reference's CPU path on a row sample, rank 0 only)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import bench
from ffn_optim_b200 import cases as C

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("case_id, gflop, mbytes", [
    ("cfg1_fp16", 2.147, 5.24), ("cfg2_bf16", 4.895, 5.60), ("cfg3_bf16", 4.295, 268.7),
    ("cfg4_bf16", 4398.0, 537.0), ("cfg5_bf16", 61572.9, 3087.0)])
def test_work_counts_of_the_configs(case_id, gflop, mbytes):
    p = C.case_problem(C.get_case(case_id))
    assert bench.flops(p) / 1e9 == pytest.approx(gflop, rel=2e-3)
    assert bench.unique_bytes(p) / 1e6 == pytest.approx(mbytes, rel=2e-3)
    # fp8 weights: one byte per weight element plus fp32 row scales
    w = p.h * p.k + p.n * p.h
    assert bench.unique_bytes(p, 1) == bench.unique_bytes(p) - w + 4 * (p.h + p.n)


@pytest.mark.parametrize("case_id", ["cfg1_fp16", "cfg2_bf16", "cfg3_bf16"])
def test_parity_rule_on_the_golden_fixture(case_id):
    fx = dict(np.load(ROOT / "tests" / "golden" / f"{case_id}.npz"))
    dtype = str(fx["dtype"])
    staged = bench.bits_to_f32(fx["staged_rational"], dtype)
    ok = bench.parity_vs_golden(staged, fx, dtype)
    assert ok["passed"] and ok["criterion"] and ok["ulp_bound_excess"] <= 0
    # every output of one row moved by 8 ulps of the output dtype: outside the 2-ulp bound
    bad = staged.copy()
    bad[0] = staged[0] * np.float32(1 + 8 * (2.0 ** -7 if dtype == "bfloat16" else 2.0 ** -10))
    bad[0][staged[0] == 0] = 1.0
    assert not bench.parity_vs_golden(bad, fx, dtype)["passed"]


def test_bits_round_trip():
    rng = np.random.Generator(np.random.PCG64(1))
    for dtype in ("bfloat16", "float16"):
        a = rng.standard_normal(1000).astype(np.float32)
        bits = bench.f32_to_bits(a, dtype)
        assert np.array_equal(bench.f32_to_bits(bench.bits_to_f32(bits, dtype), dtype), bits)


def test_kernel_names():
    assert bench.kernel_name("hslice16") == "ffn_hslice_kernel"
    assert bench.kernel_name("rowblock256") == "ffn_rowblock_kernel"
    assert bench.kernel_name("pair256x256") == "ffn_fused_kernel"


def _run_reference(extra_env):
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "cfg1_fp16",
                           "--steps", "1", "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=600)


def test_reference_arm_line():
    r = _run_reference({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    r = _run_reference({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
