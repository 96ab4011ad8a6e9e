"""Kernel-engineering tools for the agent and their executor.

Tools: ``build`` (compile / import check), ``test`` (correctness on all
shapes), ``bench`` (verified timing vs the vendor baseline), ``pmc``
(ncu counters), ``keep`` (commit the current kernel as the answer),
``revert`` (go back to the best kernel), and optionally
``list_transforms`` / ``apply_transform`` (the transform calculus). The
executor is a small state machine over (current, best) kernels and records a
per-call trace used for the tool-use shaping reward. Reference parity:
kore/agent/tools.py:60-800.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

TOOLS = [
    {"name": "build", "description": "compile/import the kernel", "parameters": {"source": "string"}},
    {"name": "test", "description": "run correctness on all shapes", "parameters": {"source": "string"}},
    {"name": "bench", "description": "verified timing vs the vendor baseline", "parameters": {"source": "string"}},
    {"name": "pmc", "description": "Nsight Compute counters of the kernel", "parameters": {"source": "string"}},
    {"name": "keep", "description": "commit this kernel as the answer", "parameters": {"source": "string"}},
    {"name": "revert", "description": "return to the best kernel so far", "parameters": {}},
]
TRANSFORM_TOOLS = [
    {"name": "list_transforms", "description": "list applicable source transforms", "parameters": {}},
    {"name": "apply_transform", "description": "apply a named transform", "parameters": {"name": "string"}},
]


@dataclass
class ToolExecutor:
    env: object
    task: object
    transforms: bool = False
    current: str = ""
    best: Optional[str] = None
    best_ms: Optional[float] = None
    kept: Optional[str] = None
    trace: List[Dict] = field(default_factory=list)

    def tools(self) -> List[Dict]:
        return TOOLS + (TRANSFORM_TOOLS if self.transforms else [])

    def call(self, name: str, args: Dict) -> Dict:
        src = args.get("source") or self.current
        self.current = src
        if name in ("build", "test", "bench", "pmc", "keep"):
            obs = self.env.step(src)
            res: Dict = {"compiled": obs.compiled, "correct": bool(obs.validation_passed),
                         "snr_db": obs.snr_by_shape or obs.snr_db}
            if obs.flagged_hack:
                res["rejected"] = obs.hack_reason
            if name in ("bench", "keep", "pmc") and obs.validation_passed:
                res.update({"wall_ms": obs.wall_by_shape, "baseline_ms": obs.baseline_by_shape})
                if obs.wall_ms and (self.best_ms is None or obs.wall_ms < self.best_ms):
                    self.best, self.best_ms = src, obs.wall_ms
            if name == "pmc" and obs.validation_passed:
                from ..verifier.pmc import collect_counters
                res["counters"] = getattr(obs, "counters", None) or {}
            if not obs.compiled:
                res["error"] = (obs.error_text or "")[-1500:]
            if name == "keep":
                self.kept = src if obs.validation_passed else self.kept
            self.trace.append({"tool": name, "ok": bool(obs.validation_passed), "ms": obs.wall_ms})
            return res
        if name == "revert":
            self.current = self.best or self.current
            self.trace.append({"tool": name, "ok": True, "ms": self.best_ms})
            return {"source": self.current}
        if name == "list_transforms":
            from ..transform.library import admissible
            return {"transforms": [t.name for t in admissible(self.current)]}
        if name == "apply_transform":
            from ..transform.library import get_transform
            t = get_transform(args.get("name", ""))
            new = t.apply(self.current) if t else None
            if new:
                self.current = new
            return {"applied": bool(new), "source": self.current}
        return {"error": f"unknown tool {name!r}"}


def tool_use_reward(trace: List[Dict], final_correct: bool) -> float:
    """Small shaping for disciplined tool use in [-0.1, 0.2]: test before
    bench, bench before keep, no repeated failing builds."""
    if not trace:
        return -0.1
    names = [t["tool"] for t in trace]
    r = 0.0
    if "test" in names and "bench" in names and names.index("test") < names.index("bench"):
        r += 0.1
    if "keep" in names and final_correct:
        r += 0.1
    fails = sum(1 for t in trace if not t.get("ok"))
    r -= 0.02 * max(0, fails - 2)
    return max(-0.1, min(0.2, r))
