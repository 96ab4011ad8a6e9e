"""Dataset assembly: grouped leakage split, win gate, capped multi-capability
mix, hard-negative floor, coverage."""
from types import SimpleNamespace as NS

from kore_b200.data.assemble import (build_multicap, coverage, dpo_with_hard_negatives, filter_trivial_wins,
                                     leakage_split)


def test_leakage_split_keeps_groups_together():
    rows = [{"task_id": f"t{i}", "family": f"f{i % 7}"} for i in range(200)]
    sp = leakage_split(rows, heldout={"t3"}, fractions=(0.6, 0.2, 0.2))
    assert sum(len(v) for v in sp.values()) == 199
    side = {}
    for name, rs in sp.items():
        for r in rs:
            assert side.setdefault(r["family"], name) == name
    assert sp == leakage_split(rows, heldout={"t3"}, fractions=(0.6, 0.2, 0.2))


def test_mix_negatives_wins_coverage():
    mix = build_multicap({"repair": [{"x": i} for i in range(10)], "qa": [{"x": i} for i in range(3)]},
                         {"repair": 4}, {"qa": 0.5})
    assert sum(1 for r in mix if r["_source"] == "repair") == 4 and len(mix) == 7
    assert all(r["_weight"] == 0.5 for r in mix if r["_source"] == "qa")
    out = dpo_with_hard_negatives([{"p": i} for i in range(50)], [{"n": i} for i in range(10)], min_frac=0.1)
    assert sum(1 for r in out if r.get("hack")) >= 0.1 * len(out) - 1e-9
    assert len(filter_trivial_wins([NS(speedup=1.5), NS(speedup=1.0), NS(speedup=None)])) == 1
    tasks = [NS(task_id="a", family="gemm"), NS(task_id="b", family="norm")]
    cov = coverage([{"task_id": "a"}, {"task_id": "a"}], tasks)
    assert cov["missing"] == ["b"] and cov["per_family"] == {"gemm": 2}
