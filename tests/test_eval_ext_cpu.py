"""fast_p family with timing-integrity gating, pass@k estimators, multi-seed
intervals, family classification / split / leave-one-family-out, champion
certification."""
import math

from kore_b200.eval.fastp import (fast_p, fast_p_at_k, fast_p_curve, gated_speedup, multi_seed, multi_seed_fast_p,
                                  pass_at_k)
from kore_b200.eval.generalization import classify, family_split, heldout_report, leave_one_family_out
from kore_b200.eval.suite import champion_verdict
from kore_b200.tasks.registry import all_tasks


def test_gating_and_fast_p():
    assert gated_speedup(1e6) == 50.0 and gated_speedup(3.0, cv_pct=12.0) == 1.0 and gated_speedup(None) == 0.0
    rs = [{"correct": True, "speedup": 2.0}, {"correct": True, "speedup": 1.2, "cv_pct": 20.0},
          {"correct": False, "speedup": 5.0}]
    assert fast_p(rs, 1.0) == 1 / 3 and fast_p(rs, 1.0, n=6) == 1 / 6
    assert fast_p_curve(rs)["fast_0.0"] == 2 / 3


def test_pass_at_k():
    assert pass_at_k(10, 0, 3) == 0.0 and pass_at_k(10, 10, 1) == 1.0
    assert abs(pass_at_k(10, 3, 1) - 0.3) < 1e-12
    exact = 1 - math.comb(7, 3) / math.comb(10, 3)
    assert abs(pass_at_k(10, 3, 3) - exact) < 1e-12
    s = {"a": [{"correct": True, "speedup": 2.0}, {"correct": False}], "b": [{"correct": True, "speedup": 0.5}] * 2}
    assert abs(fast_p_at_k(s, 1.0, 1) - 0.25) < 1e-12


def test_multi_seed():
    m, lo, hi = multi_seed([0.4, 0.5, 0.6])
    assert abs(m - 0.5) < 1e-12 and lo < 0.5 < hi
    r = multi_seed_fast_p([[{"correct": True, "speedup": 2}], [{"correct": False}]], 1.0)
    assert r["seeds"] == 2 and r["mean"] == 0.5


def test_families_split_and_lofo():
    ts = all_tasks()
    fams = {classify(t) for t in ts}
    assert {"attention", "gemm", "norm", "moe", "quant"} <= fams
    tr, ho = family_split(ts, ["attention"])
    assert ho and not set(tr) & set(ho)
    rows = [{"family": f, "x": float(i), "y": 2.0 * i + (0.1 if f == "b" else 0.0)}
            for f in ("a", "b", "c") for i in range(5)]

    def fit(train):
        n = len(train)
        mx = sum(r["x"] for r in train) / n
        my = sum(r["y"] for r in train) / n
        b = sum((r["x"] - mx) * (r["y"] - my) for r in train) / sum((r["x"] - mx) ** 2 for r in train)
        return lambda r: my + b * (r["x"] - mx)
    out = leave_one_family_out(rows, fit)
    assert out["a"]["r2"] > 0.99 and "_median" in out
    rep = heldout_report([{"task_id": ts[0].task_id, "correct": True, "speedup": 2.0}], {t.task_id: t for t in ts},
                         ["attention"])
    assert sum(v["n"] for v in rep.values()) == 1


def test_champion_verdict():
    assert champion_verdict(2.0, correct=True, speedup=1.8, cv_pct=1.0)["certified"]
    v = champion_verdict(2.0, correct=True, correct_unseen=False, speedup=1.0, cv_pct=9.0, hack_reason="cached output")
    assert not v["certified"] and len(v["reasons"]) == 4


def test_bundled_kernelbench_problems_cover_three_levels():
    from kore_b200.eval.kernelbench import _load_module, bundled_specs, spec_to_task
    specs = bundled_specs()
    assert len(specs) >= 14 and {s.level for s in specs} == {1, 2, 3}
    for s in specs:
        ns = _load_module(s)
        assert callable(ns["get_inputs"]) and ns["Model"](*ns["get_init_inputs"]()) is not None
        t = spec_to_task(s, "fp32")
        assert t.family == f"kernelbench_l{s.level}" and "def kernel(" in t.seed_src
