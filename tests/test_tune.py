"""Implementation search (reference performance/tune.py, validation/test_ffn.py SearchTests).

CPU tests drive ``search`` with simulated evaluations, as the reference's SearchTests do;
the GPU test runs the real search on the cfg1 and cfg2 workloads.
"""
import math

import pytest

from ffn_optim_b200.tune import combinations, search


def test_combinations_order_dedup_and_extra_axes():
    got = combinations(["basic", "basic"], ["basic", "streamk", "basic"])
    assert got == [{"up_impl": "basic", "down_impl": "basic"}, {"up_impl": "basic", "down_impl": "streamk"}]
    got = combinations(["basic"], ["basic", "full_load_a"], tile=[None, "pair256x256"])
    assert len(got) == 4 and got[1] == {"up_impl": "basic", "down_impl": "basic", "tile": "pair256x256"}
    with pytest.raises(ValueError):
        combinations([], ["basic"])
    with pytest.raises(ValueError):
        combinations(["basic"], ["basic"], tile=[])


def test_best_and_failure_filter():
    configs = [{"down_impl": k} for k in ("basic", "streamk", "full_load_a")]

    def evaluate(config):
        k = config["down_impl"]
        return {"status": "passed" if k != "full_load_a" else "unavailable",
                "device_median_us": {"basic": 8, "streamk": 4, "full_load_a": None}[k]}

    records, best = search(configs, evaluate)
    assert best["complete"] and best["configuration"]["down_impl"] == "streamk" and len(records) == 3
    assert records[2]["status"] == "unavailable" and records[2]["configuration"] == configs[2]


def test_dry_run_no_best():
    _, best = search([{}], lambda c: {"status": "planned"})
    assert best["configuration"] is None and best["complete"]


def test_accuracy_failure_and_bad_timings_never_win():
    def evaluate(c):
        k = c["down_impl"]
        return {"status": "accuracy_failed" if k == "streamk" else "passed",
                "device_median_us": {"streamk": 1, "basic": 10, "a": math.nan, "b": 0, "c": -3}[k]}

    _, best = search([{"down_impl": k} for k in ("streamk", "a", "b", "c", "basic")], evaluate)
    assert best["configuration"]["down_impl"] == "basic" and best["device_median_us"] == 10


def test_checkpoint_after_every_configuration_and_at_the_end():
    seen = []
    search([{"down_impl": "basic"}, {"down_impl": "streamk"}],
           lambda c: {"status": "passed", "device_median_us": 5},
           checkpoint=lambda records, best: seen.append((len(records), best["complete"])))
    assert seen == [(1, False), (2, False), (2, True)]


@pytest.mark.gpu
@pytest.mark.parametrize("case_id", ["cfg2_bf16", "cfg1_fp16"])
def test_search_on_device(case_id):
    from ffn_optim_b200 import cases as C
    from ffn_optim_b200.tune import tune_ffn

    case = C.get_case(case_id)
    x, w1, w2 = C.make_inputs(case, device="cuda")
    records, best = tune_ffn(x, w1, w2, down_candidates=("basic", "full_load_a", "full_load_b", "streamk"),
                             warmup=2, repeats=5)
    status = {r["configuration"]["down_impl"]: r["status"] for r in records}
    assert status["full_load_b"] == "unavailable" and status["basic"] == "passed"
    assert status["full_load_a"] == ("passed" if case["weight2_shape"][0] <= 512 else "not_applicable")
    passed = [r for r in records if r["status"] == "passed"]
    assert all(r["accuracy"]["passed"] and r["device_median_us"] > 0 for r in passed)
    assert best["device_median_us"] == min(r["device_median_us"] for r in passed)
