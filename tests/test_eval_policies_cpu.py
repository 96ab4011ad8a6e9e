"""Evaluation policies (seed, multi-turn model with verifier feedback,
frontier with loud unavailability) and the head-to-head comparison."""
from types import SimpleNamespace

import pytest

from kore_b200.eval import policies as P
from kore_b200.eval import vs_frontier as V
from kore_b200.tasks.registry import get_task


def _resp(src):
    return f"ANALYSIS: a\nPROPOSED_CHANGE: b\nFULL_KERNEL:\n```python\n{src}\n```\n"


def test_seed_and_multiturn_model_policy():
    t = get_task("gen_silu_bf16")
    assert P.seed_policy(t) == [t.seed_src]
    seen = []

    def gen(msgs):
        seen.append([m["role"] for m in msgs])
        return _resp(f"# turn {len(seen)}\n" + t.seed_src)

    class Env:
        def step(self, src):
            return SimpleNamespace(compiled=True, validation_passed=True, snr_db=60.0, wall_ms=1.0, speedup=1.0,
                                   error_text=None, speedup_by_shape={}, cv_pct=1.0, flagged_hack=False,
                                   hack_reason=None, infra_error=None, reward=0.0)
    srcs = P.model_policy(gen, turns=3, env_factory=lambda task: Env())(t)
    assert len(srcs) == 3 and srcs[0].startswith("# turn 1")
    assert seen[-1][-2:] == ["assistant", "user"]                # feedback before the last turn
    assert len(P.model_policy(gen, turns=3)(t)) == 1              # no environment: one shot


def test_frontier_policy_is_loud_when_unavailable():
    t = get_task("gen_silu_bf16")
    with pytest.raises(P.FrontierUnavailable):
        P.frontier_policy()

    class Down:
        def generate(self, m):
            raise ConnectionError("refused")
    with pytest.raises(P.FrontierUnavailable):
        P.frontier_policy(Down())(t)

    class Empty:
        def generate(self, m):
            return "  "
    with pytest.raises(P.FrontierUnavailable):
        P.frontier_policy(Empty())(t)


def test_winner_rules_and_compare():
    c = lambda s: {"task_id": "t", "correct": True, "speedup": s}         # noqa: E731
    bad = {"task_id": "t", "correct": False, "speedup": 0.0}
    assert V.winner_for_task(c(1.5), c(1.0)) == "ours"
    assert V.winner_for_task(c(1.0), c(1.01)) == "tie"
    assert V.winner_for_task(bad, c(0.5)) == "theirs"
    assert V.winner_for_task(bad, bad) == "tie"
    assert V.winner_for_task(c(1.0), None) == "unavailable"
    res = V.compare([c(2.0), c(1.0), bad, c(1.3)], [c(1.0), c(1.5), bad, None])
    assert (res["wins"], res["losses"], res["ties"], res["unavailable"]) == (1, 1, 1, 1)
    assert res["win_rate"] == 0.5 and 0 <= res["win_rate_ci95"][0] <= 0.5 <= res["win_rate_ci95"][1] <= 1
    assert "| fast_p |" in V.format_report(res)


def test_head_to_head_counts_unavailable_frontier(monkeypatch):
    tasks = [get_task("gen_silu_bf16"), get_task("gen_relu_bf16")]
    import kore_b200.eval.bakeoff as B

    def fake_eval(policy, ts, envf, budget):
        return [dict(policy(t), task_id=t.task_id) for t in ts]
    monkeypatch.setattr(B, "evaluate_policy", fake_eval)

    def theirs(t):
        if t.task_id == "gen_relu_bf16":
            raise P.FrontierUnavailable("down")
        return {"correct": True, "speedup": 1.0}
    res = V.head_to_head(lambda t: {"correct": True, "speedup": 1.5}, theirs, tasks, None)
    assert res["wins"] == 1 and res["unavailable"] == 1 and res["losses"] == 0
