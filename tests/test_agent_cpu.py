"""Agent harness on a scripted environment: Kevin credit, phase switch,
reseed escape, per-turn physics trace, bench frontier feedback, transform
tools with an epsilon budget, family-keyed few-shot retrieval, reflections."""
import json
import re

from kore_b200.agent.format import (episode_to_chat, parse_reflection, parse_tool_calls, reflection_is_grounded,
                                    render_tool_call)
from kore_b200.agent.harness import AgentHarness, WinsKB
from kore_b200.agent.tools import ToolExecutor, agent_tool_schemas
from kore_b200.reward.reward import Observation
from kore_b200.tasks.registry import get_task

TASK = get_task("gemm_bf16")


class FakeEnv:
    """Correct iff the source contains 'OK'; time = 1 / (1 + number of 'FAST')."""
    task = TASK

    def step(self, src):
        ok = "OK" in src
        ms = 1.0 / (1 + src.count("FAST")) if ok else None
        return Observation(compiled=True, snr_db=60.0 if ok else 5.0, wall_ms=ms, baseline_ms=1.0 if ok else None,
                           wall_by_shape={"primary": ms} if ok else {}, baseline_by_shape={"primary": 1.0} if ok else {},
                           snr_by_shape={"primary": 60.0 if ok else 5.0}, validation_passed=ok, dtype="bf16")


class Script:
    def __init__(self, turns):
        self.turns = list(turns)

    def generate(self, msgs):
        return self.turns.pop(0) if self.turns else ""


def call(name, src=None, **kw):
    args = dict(kw)
    if src is not None:
        args["source"] = src
    return render_tool_call(name, args)


def test_formats():
    t = "<reflection>the test failed: wrong output</reflection>\n" + call("test", "x")
    assert parse_tool_calls(t) == [{"name": "test", "arguments": {"source": "x"}}]
    assert parse_reflection(t).startswith("the test failed")
    assert reflection_is_grounded(parse_reflection(t), {"correct": False})
    assert not reflection_is_grounded("nice weather", {"correct": False})
    chat = episode_to_chat([{"role": "assistant", "content": "<think>x</think>answer"}])
    assert chat[0]["content"] == "answer"
    assert {s["function"]["name"] for s in agent_tool_schemas(True)} >= {"bench", "apply_transform"}


def test_episode_credit_phase_and_trace():
    pol = Script([call("test", "bad"),
                  "<reflection>test failed, incorrect</reflection>" + call("test", "OK"),
                  call("bench", "OK FAST"),
                  call("keep", "OK FAST")])
    h = AgentHarness(FakeEnv(), TASK, max_turns=6)
    ep = h.run(pol)
    assert ep.turn_correct == [False, True, True, True]
    assert len(ep.turn_rewards) == len(ep.turn_speedups) == len(ep.turn_phis) == len(ep.codes) == 4
    assert ep.turn_speedups[0] is None and ep.turn_speedups[1] is None      # only benched turns
    assert ep.turn_speedups[2] is not None and ep.turn_speedups[2] > 1.5
    assert ep.best_correct == "OK FAST" and h.phase == "optimize"
    assert "FASTER" in ep.messages[0]["content"]
    assert ep.reflections == 1 and ep.tool_reward > 0


def test_bench_frontier_fields():
    ex = ToolExecutor(FakeEnv(), TASK, current="OK")
    r1 = ex.call("bench", {"source": "OK FAST"})
    assert r1["improved_frontier"] and r1["delta_vs_best"] is None
    r2 = ex.call("bench", {"source": "OK"})
    assert not r2["improved_frontier"] and r2["delta_vs_best"] < 0
    assert r2["best_speedup_so_far"] == r1["speedup"]
    r3 = ex.call("bench", {"source": "OK FAST FAST"})
    assert r3["improved_frontier"] and ex.best == "OK FAST FAST"


def test_reseed_keeps_best():
    turns = [call("test", "OK")] + [call("test", "bad")] * 4
    h = AgentHarness(FakeEnv(), TASK, max_turns=5, reseed_patience=3)
    ep = h.run(Script(turns))
    assert ep.reseeds == 1 and ep.best_correct == "OK"
    assert any("reset to the seed" in m["content"] for m in ep.messages if m["role"] == "user")


def test_transform_tools_spend_budget():
    ex = ToolExecutor(FakeEnv(), TASK, transforms=True, current=TASK.seed_src)
    lst = ex.call("list_transforms", {})
    names = [t["name"] for t in lst["transforms"]]
    assert any(n.startswith("set_num_stages") for n in names)
    before = ex.call("list_transforms", {})["budget_remaining"]
    r = ex.call("apply_transform", {"name": "downcast_dtype", "params": {"to": "bf16"}})
    if r["applied"]:
        assert r["budget_remaining"] < before
    bad = ex.call("apply_transform", {"name": "no_such"})
    assert not bad["applied"] and "unknown" in bad["reason"]


class Win:
    def __init__(self, family, dtype, speedup, k):
        self.family, self.dtype, self.speedup, self.final_kernel, self.operation = family, dtype, speedup, k, family


def test_wins_kb_same_family_only():
    kb = WinsKB([Win("gemm", "bf16", 2.0, "KGEMM"), Win("norm", "bf16", 5.0, "KNORM")])
    assert [w.final_kernel for w in kb.examples("gemm", "bf16")] == ["KGEMM"]
    assert kb.examples("attention", "bf16") == []


def test_tool_call_validation_and_reward_breakdown():
    from kore_b200.agent.tools import tool_use_breakdown, validate_tool_call
    assert validate_tool_call("bench", {"source": "x"})["error"] is None
    assert validate_tool_call("benchmark", {})["valid_name"] is False
    v = validate_tool_call("bench", {"src": "x"})
    assert v["valid_name"] and not v["valid_params"] and "unknown parameter" in v["error"]
    assert "must be a string" in validate_tool_call("bench", {"source": 3})["error"]
    assert "missing" in validate_tool_call("apply_transform", {})["error"]
    assert validate_tool_call("revert", None)["error"] is None
    trace = [{"tool": "build", "ok": False, "error": "ptxas error: shared memory overflow in kernel"},
             {"tool": "test", "ok": True}, {"tool": "bench", "ok": True}, {"tool": "keep", "ok": True},
             {"tool": "benchmark", "ok": False, "valid_name": False, "valid_params": False}]
    good = tool_use_breakdown(trace, True, reflections=["the shared memory overflow came from BLOCK 256"], turns=2,
                              decisions=[{"action": "keep", "right": True}])
    bad = tool_use_breakdown(trace, True, reflections=["nice weather today"], turns=2,
                             decisions=[{"action": "keep", "right": False}])
    assert good["order"] == 1.0 and good["commit"] == 1.0 and good["name"] == 0.8
    assert good["reflection"] > bad["reflection"] and good["decisions"] == 1.0 and bad["decisions"] == -1.0
    assert -0.1 <= bad["total"] < good["total"] <= 0.25
    assert tool_use_breakdown([], False)["total"] == -0.1


def test_executor_rejects_bad_calls_and_tracks_decisions():
    from types import SimpleNamespace

    from kore_b200.agent.tools import ToolExecutor
    from kore_b200.tasks.registry import get_task
    t = get_task("gen_silu_bf16")

    class Env:
        def step(self, src):
            ok = "bad" not in src
            return SimpleNamespace(compiled=True, validation_passed=ok, wall_ms=1.0 if ok else None, snr_db=60.0,
                                   flagged_hack=False, error_text=None if ok else "SNR 2 dB mismatch",
                                   wall_by_shape={"primary": 1.0}, baseline_by_shape={"primary": 1.0},
                                   speedup_by_shape={"primary": 1.0}, counters=None)
    ex = ToolExecutor(Env(), t, current=t.seed_src)
    r = ex.call("frobnicate", {})
    assert "unknown tool" in r["error"] and ex.trace[-1]["valid_name"] is False
    ex.call("test", {"source": "bad kernel"})
    assert "mismatch" in ex.trace[-1]["error"]
    ex.call("revert", {})
    ex.call("keep", {"source": t.seed_src})
    assert [d["action"] for d in ex.decisions] == ["revert", "keep"]
