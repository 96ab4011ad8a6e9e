"""Multi-turn tool-use loop over the kernel environment.

render -> generate -> parse reflection and tool calls -> execute -> tool
results back into the conversation, until ``keep`` or the turn budget.

* Kevin credit: the episode is scored by its best correct candidate (by
  reward), not its last turn; ``turn_rewards`` / ``turn_correct`` are recorded
  per assistant turn, unrounded.
* Phase switch: the system prompt asks for correctness until the first
  correct kernel, then for speed.
* Reseed escape: after ``reseed_patience`` turns without a better correct
  candidate the working lineage restarts from the seed; the best kernel is
  kept.
* Per-turn physics trace, index-aligned with ``turn_rewards``:
  ``turn_speedups`` (measured, benched correct turns only), ``turn_phis``
  (roofline potential for potential-based shaping) and ``codes``.
* ``WinsKB`` retrieves prior wins of the same (family, dtype) as few-shot
  examples; never another family's.

Reference behaviour: kore/agent/harness.py:52-436.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

from .format import (build_agent_system_prompt, format_tool_result, parse_reflection, parse_tool_calls,
                     reflection_is_grounded)
from .tools import EVAL_TOOLS, ToolExecutor, tool_use_breakdown


@dataclass
class Episode:
    messages: List[dict]
    turn_rewards: List[float] = field(default_factory=list)
    turn_correct: List[bool] = field(default_factory=list)
    codes: List[str] = field(default_factory=list)
    turn_speedups: List[Optional[float]] = field(default_factory=list)
    turn_phis: List[Optional[float]] = field(default_factory=list)
    best_correct: Optional[str] = None
    best_ms: Optional[float] = None
    best_speedup: Optional[float] = None
    tool_reward: float = 0.0
    tool_breakdown: Dict[str, float] = field(default_factory=dict)
    reflections: int = 0                                   # reflections grounded in the last tool result
    reflection_texts: List[str] = field(default_factory=list)
    reseeds: int = 0

    @property
    def turn_codes(self) -> List[str]:
        return self.codes

    def to_record(self, task_id: str):
        from .schema import AgenticTrajectoryRecord
        return AgenticTrajectoryRecord(task_id, self.messages, [], list(self.turn_rewards), list(self.turn_correct),
                                       self.best_correct, self.best_speedup)


AgentEpisode = Episode


class WinsKB:
    """Few-shot retriever over WinRecords keyed by (family, dtype)."""

    def __init__(self, records=()):
        self.by_key: Dict[tuple, list] = {}
        for r in records:
            self.by_key.setdefault(self._key(r), []).append(r)

    @staticmethod
    def _key(r) -> tuple:
        fam = getattr(r, "family", None) or getattr(r, "operation", "") or ""
        return (fam, getattr(r, "dtype", None) or "")

    def examples(self, family: str, dtype: str = "", k: int = 1) -> List:
        rs = self.by_key.get((family, dtype), []) or (self.by_key.get((family, ""), []) if not dtype else [])
        return sorted(rs, key=lambda r: -(getattr(r, "speedup", 0) or 0))[:k]


class AgentHarness:
    def __init__(self, env, task, *, max_turns: int = 8, transforms: bool = False, kb: Optional[WinsKB] = None,
                 reward_fn: Optional[Callable] = None, reseed_patience: int = 3, arch: Optional[str] = None):
        self.env, self.task = env, task
        self.max_turns = max_turns
        self.exec = ToolExecutor(env, task, transforms=transforms, current=task.seed_src)
        self.kb = kb
        self.reward_fn = reward_fn
        self.reseed_patience = reseed_patience
        self.arch = arch
        self.phase = "correctness"

    def _system(self) -> str:
        return build_agent_system_prompt(self.exec.tools(), arch=self.arch, phase=self.phase)

    def initial_messages(self) -> List[dict]:
        from ..policy.format import build_task_prompt
        user = build_task_prompt(self.task)
        if self.kb:
            fam = getattr(self.task, "family", "") or getattr(self.task, "operation", "")
            for ex in self.kb.examples(fam, getattr(self.task, "dtype", "")):
                user += (f"\n\nA previous winning kernel for a {fam} task ({(ex.speedup or 0):.2f}x):\n"
                         f"{ex.final_kernel}")
        return [{"role": "system", "content": self._system()}, {"role": "user", "content": user}]

    def run(self, policy) -> Episode:
        """Drive the tool loop. The per-turn lists have one entry per assistant
        turn (the best evaluation among that turn's calls; 0 and incorrect
        for a turn without one), aligned with the policy's generations."""
        msgs = self.initial_messages()
        ep = Episode(messages=msgs)
        ex = self.exec
        stall, last_res, best_key = 0, None, None
        for _ in range(self.max_turns):
            resp = policy.generate(msgs)
            msgs.append({"role": "assistant", "content": resp})
            refl = parse_reflection(resp)
            if refl:
                ep.reflection_texts.append(refl)
            if reflection_is_grounded(refl, last_res):
                ep.reflections += 1
            calls = parse_tool_calls(resp)
            if not calls:
                from ..policy.format import parse_response
                k = parse_response(resp).get("kernel")
                calls = [{"name": "keep", "arguments": {"source": k}}] if k else []
            if not calls:
                self._record(ep, None)
                break
            stop, turn_best = False, None
            for c in calls:
                res = ex.call(c["name"], c["arguments"])
                last_res = res
                msgs.append({"role": "tool", "content": format_tool_result(c["name"], res)})
                if c["name"] in EVAL_TOOLS:
                    ok = ex.candidate_correct
                    r = self.reward_fn(res) if self.reward_fn else (ex.candidate_reward or 0.0)
                    cand = (ok, r, ex.current, ex.candidate_speedup, ex.candidate_phi)
                    if turn_best is None or (ok, r) > (turn_best[0], turn_best[1]):
                        turn_best = cand
                if c["name"] == "keep" and ex.candidate_correct:
                    stop = True
            self._record(ep, turn_best)
            if turn_best is not None and turn_best[0]:
                if self.phase == "correctness":          # first correct kernel: optimise from here on
                    self.phase = "optimize"
                    msgs[0] = {"role": "system", "content": self._system()}
                key = turn_best[1]
                if best_key is None or key > best_key:
                    best_key, stall = key, 0
                else:
                    stall += 1
            else:
                stall += 1
            if stop:
                break
            if stall >= self.reseed_patience:
                ex.reseed()
                ep.reseeds += 1
                stall = 0
                msgs.append({"role": "user", "content": "No progress for several turns: the working kernel was "
                                                        "reset to the seed (your best kernel is kept). Try a "
                                                        "different approach."})
        ep.best_correct = ex.kept or ex.best_reward_src or ex.best
        ep.best_ms = ex.best_ms
        ep.best_speedup = ex.best_speedup
        n_turns = len(ep.turn_rewards)
        ep.tool_breakdown = tool_use_breakdown(ex.trace, ep.best_correct is not None,
                                               reflections=ep.reflection_texts, turns=n_turns,
                                               decisions=ex.decisions)
        ep.tool_reward = ep.tool_breakdown["total"]
        return ep

    def _record(self, ep: Episode, best) -> None:
        if best is None:
            ep.turn_correct.append(False)
            ep.turn_rewards.append(0.0)
            ep.codes.append(self.exec.current)
            ep.turn_speedups.append(None)
            ep.turn_phis.append(None)
            return
        ok, r, code, sp, phi = best
        ep.turn_correct.append(bool(ok))
        ep.turn_rewards.append(float(r))
        ep.codes.append(code)
        ep.turn_speedups.append(sp if ok else None)
        ep.turn_phis.append(phi if ok else None)
