"""CPU tests: transform calculus, search, value model, open-ended curriculum,
task minter, eval statistics/gates, data hygiene, agent tool parsing."""
import json
import math
import random

import numpy as np
import pytest

SRC = """import triton
import triton.language as tl

@triton.jit
def k(X, Y, N, BLOCK: tl.constexpr):
    x = tl.exp(tl.load(X))

def run(x):
    k[(1,)](x, x, 1, BLOCK=128, num_warps=4)
"""


def test_transform_sequence_and_budget():
    from kore_b200.transform.calculus import EpsBudget, apply_sequence
    from kore_b200.transform.library import LIBRARY, admissible, get_transform
    names = {a.transform.name for a in admissible(SRC)}
    assert {"retile_block", "exp_to_exp2", "set_num_warps"} <= names
    out, applied = apply_sequence(SRC, [get_transform("retile_block(f=x2,name=BLOCK)"),
                                        get_transform("set_num_warps(n=8)")])
    assert "BLOCK=256" in out and "num_warps=8" in out
    assert applied == ["retile_block(f=x2,name=BLOCK)", "set_num_warps(n=8)"]
    b = EpsBudget(total=0.0)
    approx = [t for t in LIBRARY if t.kind == "approx"][0]
    assert not b.can_afford(approx)


def test_successive_halving_picks_best():
    from kore_b200.search.bandit import Budget, successive_halving
    rng = random.Random(0)
    means = {"a": 1.0, "b": 2.0, "c": 1.5, "d": 0.5}
    best = successive_halving(list(means), lambda a: means[a] + rng.gauss(0, 0.05), Budget(64))
    assert best == "b"


def test_puct_search_improves():
    from kore_b200.search.alphakernel import search

    def ev(src):
        import re
        m = re.search(r"BLOCK=(\d+)", src)
        return 1.0 + math.log2(int(m.group(1))) / 10 if m else None
    r = search(SRC, ev, budget=12)
    assert r.best_score > ev(SRC) and r.evaluated <= 12 and r.path


def test_value_model_roundtrip_and_rank():
    from kore_b200.value.model import ValueModel, features, rank_candidates
    srcs = [SRC.replace("BLOCK=128", f"BLOCK={b}") for b in (32, 64, 128, 256, 512, 1024)]
    F = np.stack([features(s) for s in srcs])
    ls = np.array([math.log2(b) / 10 for b in (32, 64, 128, 256, 512, 1024)])
    m = ValueModel("v1").fit(F, np.ones(6), np.ones(6), ls, pairs=[(5, 0), (4, 1), (3, 2)])
    m2 = ValueModel.from_json(m.to_json())
    assert np.allclose(m.predict(F)["utility"], m2.predict(F)["utility"])
    assert rank_candidates(m2, srcs)[0] == 5


def test_curriculum_deterministic_and_informative():
    from kore_b200.openended.core import CurriculumController, coevolve
    a, b = CurriculumController(seed=3), CurriculumController(seed=3)
    assert a.next_task_id(4) == b.next_task_id(4)
    tid = a.next_task_id(1)[0]
    for _ in range(10):
        a.record(tid, True)
    e = a.archive.entries[tid]
    assert e.informativeness < 0.5                       # solved tasks stop being informative
    log = coevolve(CurriculumController(), lambda t: (True, 1.2), rounds=2, batch=2)
    assert len(log) == 4


def test_minter_gate():
    from kore_b200.openended.minter import construction_gate, mint
    from kore_b200.tasks.ops_library import SPECS
    assert construction_gate(lambda a, b: b) == "ignores input a"
    assert construction_gate(lambda a, b: a / 0 * 0) is not None
    made = mint(2, seed=1)
    assert len(made) == 2 and all(t in SPECS for t in made)


def test_eval_stats_and_gates(tmp_path):
    from kore_b200.eval.bakeoff import assert_no_leakage
    from kore_b200.eval.gates import retention_gate, run_retention_suite
    from kore_b200.eval.metrics import bootstrap_ci, fast_p, sign_test, wilcoxon
    res = [{"correct": True, "speedup": 1.3}, {"correct": True, "speedup": 0.9}, {"correct": False, "speedup": 5}]
    assert fast_p(res, 1.0) == pytest.approx(1 / 3) and fast_p(res, 0.5) == pytest.approx(2 / 3)
    a = [1.0 + 0.1 * i for i in range(20)]
    b = [x - 0.5 for x in a]
    m, lo, hi = bootstrap_ci(a, b)
    assert m == pytest.approx(0.5) and lo <= 0.5 <= hi
    assert sign_test(a, b) < 1e-4 and wilcoxon(a, b) < 1e-3
    assert sign_test(a, a) == 1.0
    assert retention_gate({"mmlu": 0.6}, {"mmlu": 0.59}, 0.005).passed is False
    assert retention_gate({"mmlu": 0.6}, {"mmlu": 0.598}, 0.005).passed
    suite = tmp_path / "s.jsonl"
    suite.write_text(json.dumps({"prompt": "2+2", "answer": "4"}) + "\n" + json.dumps({"prompt": "x", "answer": "y"}) + "\n")
    sc = run_retention_suite(lambda p: "the answer is 4", {"toy": str(suite)}, cache_path=str(tmp_path / "c.json"))
    assert sc["toy"] == 0.5
    with pytest.raises(AssertionError):
        assert_no_leakage(["a", "b"], ["b"])


def test_hygiene_dedup_decontaminate():
    from kore_b200.data.hygiene import decontaminate, dedup, quality_ok
    base = "def f(x):\n    return x * 2 + 1  # doubling then increment of the value\n"
    items = [base, base + " ", "completely different text about kernels and tiles and warps"]
    assert len(dedup(items)) == 2
    assert len(decontaminate(items, [base])) == 1
    assert quality_ok("import torch\n" + "x = 1\n") in (True, False)


def test_agent_tool_call_parsing():
    from kore_b200.agent.format import format_tool_result, parse_tool_calls
    txt = 'I will test.\n<tool_call>{"name": "test", "arguments": {"source": "x"}}</tool_call>'
    calls = parse_tool_calls(txt)
    assert calls and calls[0]["name"] == "test" and calls[0]["arguments"]["source"] == "x"
    assert "test" in format_tool_result("test", {"correct": True})


def test_eval_suites(tmp_path):
    import types
    from kore_b200.data.schemas import WinRecord
    from kore_b200.eval.suite import KOREBENCH_V1, champion_reeval, head_to_head, korebench, write_report
    from kore_b200.tasks.ops_library import SPECS
    from kore_b200.tasks.registry import get_task
    assert all(t in SPECS for t in KOREBENCH_V1)

    class Env:
        def __init__(self, t):
            self.t = t

        def step(self, src):
            fast = "fast" in src
            return types.SimpleNamespace(validation_passed=True, compiled=True, wall_ms=1.0,
                                         wall_by_shape={"primary": 1.0 if fast else 2.0},
                                         baseline_by_shape={"primary": 1.5}, cv_by_shape=None)
    tasks = [get_task(t) for t in KOREBENCH_V1[:3]]
    h = head_to_head(lambda t: ["fast"], lambda t: ["slow"], tasks, Env)
    assert h["a_win_rate"] == 1.0
    kb = korebench(lambda t: ["fast"], Env, KOREBENCH_V1[:4])
    assert kb["fast_1.0"] == 1.0 and kb["fast_1.5"] == 1.0
    ch = champion_reeval([WinRecord(KOREBENCH_V1[0], [], 1, 1, 3.0, final_kernel="slow")],
                         {t.task_id: t for t in tasks}, Env, min_speedup=1.0)
    assert ch[0]["kept"] is False and ch[0]["claimed"] == 3.0
    txt = write_report(str(tmp_path / "r.md"), "eval", {"korebench": kb})
    assert "fast_1.0" in txt


def test_minted_task_materializes(tmp_path):
    from kore_b200.openended.minter import materialize, mint
    tid = mint(1, seed=5)[0]
    d = materialize(tid, str(tmp_path))
    from kore_b200.tasks.base import Task
    t = Task.from_dir(d)
    from kore_b200.tasks.ops_library import SPECS
    assert t.task_id == tid and t.shape("primary").dims == SPECS[tid].shapes["primary"]
