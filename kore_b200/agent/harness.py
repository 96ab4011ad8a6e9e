"""Multi-turn agent loop: render -> generate -> parse tool calls -> execute
-> tool results back into the conversation, until ``keep`` or the turn
budget. The episode is scored by its best correct kernel; per-turn rewards,
correctness, speedups, codes and potentials are traced for GRPO credit.
``WinsKB`` retrieves few-shot winning trajectories for the same operation.
Reference parity: kore/agent/harness.py:52-436."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

from .format import build_agent_system_prompt, format_tool_result, parse_tool_calls
from .tools import ToolExecutor, tool_use_reward


@dataclass
class Episode:
    messages: List[dict]
    turn_rewards: List[float] = field(default_factory=list)
    turn_correct: List[bool] = field(default_factory=list)
    codes: List[str] = field(default_factory=list)
    best_correct: Optional[str] = None
    best_ms: Optional[float] = None
    tool_reward: float = 0.0


class WinsKB:
    """Few-shot retriever over WinRecords keyed by operation."""

    def __init__(self, records=()):
        self.by_op: Dict[str, list] = {}
        for r in records:
            self.by_op.setdefault(r.operation or "", []).append(r)

    def examples(self, operation: str, k: int = 1) -> List:
        rs = sorted(self.by_op.get(operation, []), key=lambda r: -(r.speedup or 0))
        return rs[:k]


class AgentHarness:
    def __init__(self, env, task, *, max_turns: int = 8, transforms: bool = False, kb: Optional[WinsKB] = None,
                 reward_fn: Optional[Callable] = None):
        self.env, self.task = env, task
        self.max_turns = max_turns
        self.exec = ToolExecutor(env, task, transforms=transforms, current=task.seed_src)
        self.kb = kb
        self.reward_fn = reward_fn

    def initial_messages(self) -> List[dict]:
        from ..policy.format import build_task_prompt
        sys_p = build_agent_system_prompt(self.exec.tools())
        user = build_task_prompt(self.task)
        if self.kb:
            for ex in self.kb.examples(self.task.operation):
                user += f"\n\nA previous winning kernel for {ex.operation} ({ex.speedup:.2f}x):\n{ex.final_kernel}"
        return [{"role": "system", "content": sys_p}, {"role": "user", "content": user}]

    def run(self, policy) -> Episode:
        """Drive the tool loop. ``turn_rewards`` / ``turn_correct`` / ``codes``
        have one entry per assistant turn (the best evaluation among that
        turn's test/bench/keep calls; 0 and incorrect for a turn without one),
        so they align with the policy's recorded generations."""
        msgs = self.initial_messages()
        ep = Episode(messages=msgs)
        for _ in range(self.max_turns):
            resp = policy.generate(msgs)
            turn_best = None
            msgs.append({"role": "assistant", "content": resp})
            calls = parse_tool_calls(resp)
            if not calls:
                from ..policy.format import parse_response
                k = parse_response(resp).get("kernel")
                calls = [{"name": "keep", "arguments": {"source": k}}] if k else []
            if not calls:
                ep.turn_correct.append(False)
                ep.turn_rewards.append(0.0)
                ep.codes.append(self.exec.current)
                break
            stop = False
            for c in calls:
                res = self.exec.call(c["name"], c["arguments"])
                msgs.append({"role": "tool", "content": format_tool_result(c["name"], res)})
                if c["name"] in ("test", "bench", "keep"):
                    ok = bool(res.get("correct"))
                    r = self.reward_fn(res) if self.reward_fn else (0.3 if ok else 0.0)
                    if turn_best is None or (ok, r) > (turn_best[0], turn_best[1]):
                        turn_best = (ok, r, self.exec.current)
                if c["name"] == "keep":
                    stop = True
            ok, r, code = turn_best if turn_best is not None else (False, 0.0, self.exec.current)
            ep.turn_correct.append(ok)
            ep.turn_rewards.append(r)
            ep.codes.append(code)
            if stop:
                break
        ep.best_correct = self.exec.kept or self.exec.best
        ep.best_ms = self.exec.best_ms
        ep.tool_reward = tool_use_reward(self.exec.trace, ep.best_correct is not None)
        return ep
