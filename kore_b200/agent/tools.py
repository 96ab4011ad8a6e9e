"""Kernel-engineering tools for the agent and their executor.

Base tools: ``build`` (compile / import check), ``test`` (correctness on every
shape), ``bench`` (verified timing against the vendor baseline), ``pmc``
(Nsight Compute counters), ``keep`` (commit a kernel as the answer),
``revert`` (return to the best kernel). Opt-in transform tools:
``list_transforms`` (the typed rewrites admissible for the working kernel under
the episode's remaining epsilon budget) and ``apply_transform`` (one rewrite
with budget accounting; an inadmissible move is refused and the source left
unchanged). The executor is the episode's state machine:

* it grades every evaluated candidate with the system's reward
  (``compute_kernel_reward``; mode from ``KORE_REWARD_MODE``, default
  ``speedup``) and keeps the best correct candidate by reward (the Kevin
  scoring key) and, separately, the measured-speedup frontier;
* a ``bench`` result carries ``best_speedup_so_far``, ``delta_vs_best`` and
  ``improved_frontier`` (the frontier snapshotted before this candidate);
* per evaluation it records ``candidate_speedup`` (only for a benched correct
  kernel) and ``candidate_phi`` (the roofline potential for shaping);
* ``reseed`` restarts the working lineage from the seed while keeping the best
  kernel and resetting the epsilon budget;
* ``trace`` feeds the tool-use shaping reward.

Tool schemas are OpenAI-style function descriptions.
Reference behaviour: kore/agent/tools.py:60-800.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional


def _fn(name: str, desc: str, props: Dict[str, dict], required=()) -> Dict:
    return {"type": "function", "function": {"name": name, "description": desc,
                                             "parameters": {"type": "object", "properties": props,
                                                            "required": list(required)}}}


_SRC = {"source": {"type": "string", "description": "the complete kernel module (defaults to the working kernel)"}}
TOOL_SCHEMAS = [
    _fn("build", "Compile / import the kernel module and report errors.", _SRC),
    _fn("test", "Run the correctness check (SNR against the fp32 reference) on every shape.", _SRC),
    _fn("bench", "Verified timing against the vendor baseline, with the speedup frontier of this episode.", _SRC),
    _fn("pmc", "Nsight Compute counters of the kernel (DRAM / tensor-pipe utilisation, stalls).", _SRC),
    _fn("keep", "Commit this kernel as the final answer (it must be correct).", _SRC),
    _fn("revert", "Make the best kernel of this episode the working kernel again.", {}),
]
TRANSFORM_SCHEMAS = [
    _fn("list_transforms", "Typed source rewrites admissible for the working kernel under the remaining "
                           "approximation budget.", {}),
    _fn("apply_transform", "Apply one typed rewrite (with its parameters) to the working kernel.",
        {"name": {"type": "string", "description": "transform family or family(k=v,...)"},
         "params": {"type": "object", "description": "parameters of the family"}}, required=("name",)),
]
# flat schema list kept for callers that want name / description only
TOOLS = [{"name": t["function"]["name"], "description": t["function"]["description"],
          "parameters": {k: v["type"] for k, v in t["function"]["parameters"]["properties"].items()}}
         for t in TOOL_SCHEMAS]
TRANSFORM_TOOLS = [{"name": t["function"]["name"], "description": t["function"]["description"],
                    "parameters": {k: v["type"] for k, v in t["function"]["parameters"]["properties"].items()}}
                   for t in TRANSFORM_SCHEMAS]
EVAL_TOOLS = ("build", "test", "bench", "pmc", "keep")


def agent_tool_schemas(transforms: bool = False) -> List[Dict]:
    return TOOL_SCHEMAS + (TRANSFORM_SCHEMAS if transforms else [])


_JSON_TYPES = {"string": str, "object": dict, "number": (int, float), "integer": int, "boolean": bool,
               "array": list}


def validate_tool_call(name: str, arguments, schemas: Optional[List[Dict]] = None) -> Dict:
    """Check a parsed call against the OpenAI-style schemas: a known tool
    name, an object of arguments, every required parameter present, no
    unknown parameter, each of the declared JSON type. Returns
    {"valid_name", "valid_params", "error"} (error None when valid)."""
    schemas = schemas if schemas is not None else agent_tool_schemas(True)
    by_name = {s["function"]["name"]: s["function"]["parameters"] for s in schemas}
    if name not in by_name:
        return {"valid_name": False, "valid_params": False,
                "error": f"unknown tool {name!r}; available: {', '.join(sorted(by_name))}"}
    if arguments is None:
        arguments = {}
    if not isinstance(arguments, dict):
        return {"valid_name": True, "valid_params": False, "error": "arguments must be a JSON object"}
    spec = by_name[name]
    props = spec.get("properties", {})
    missing = [r for r in spec.get("required", []) if r not in arguments]
    if missing:
        return {"valid_name": True, "valid_params": False, "error": f"missing required parameter(s): {missing}"}
    unknown = [k for k in arguments if k not in props]
    if unknown:
        return {"valid_name": True, "valid_params": False,
                "error": f"unknown parameter(s) {unknown}; {name} takes {sorted(props) or 'none'}"}
    for k, v in arguments.items():
        t = _JSON_TYPES.get(props[k].get("type", ""))
        if t is not None and v is not None and not isinstance(v, t):
            return {"valid_name": True, "valid_params": False,
                    "error": f"parameter {k!r} must be a {props[k]['type']}"}
    return {"valid_name": True, "valid_params": True, "error": None}


@dataclass
class ToolExecutor:
    env: object
    task: object
    transforms: bool = False
    current: str = ""
    best: Optional[str] = None                 # fastest correct kernel by measured time
    best_ms: Optional[float] = None
    best_reward: Optional[float] = None        # Kevin key: best correct candidate by reward
    best_reward_src: Optional[str] = None
    best_speedup: Optional[float] = None       # measured-speedup frontier
    kept: Optional[str] = None
    candidate_speedup: Optional[float] = None  # of the last evaluation (benched + correct only)
    candidate_phi: Optional[float] = None
    candidate_reward: Optional[float] = None
    candidate_correct: bool = False
    trace: List[Dict] = field(default_factory=list)
    reward_mode: str = field(default_factory=lambda: os.environ.get("KORE_REWARD_MODE", "speedup"))
    budget: object = None                      # per-episode epsilon budget of the transform tools
    seed_src: str = ""
    decisions: List[Dict] = field(default_factory=list)   # keep / revert decisions and whether they were right

    def __post_init__(self):
        self.seed_src = self.seed_src or self.current

    def tools(self) -> List[Dict]:
        return TOOLS + (TRANSFORM_TOOLS if self.transforms else [])

    def schemas(self) -> List[Dict]:
        return agent_tool_schemas(self.transforms)

    # ------------------------------------------------------------------ grading
    def _grade(self, obs, src: str):
        try:
            from ..reward.physics import compute_kernel_reward
            rr = compute_kernel_reward(obs, src, self.task, mode=self.reward_mode,
                                       dtype=getattr(self.task, "dtype", "fp32"))
            return float(rr.reward), bool(rr.correct), rr.speedup
        except Exception:  # noqa: BLE001 - a reward failure must not end the episode
            ok = bool(getattr(obs, "validation_passed", False))
            return (0.3 if ok else 0.0), ok, None

    def _phi(self, obs) -> Optional[float]:
        try:
            from ..reward.whitebox import phi_potential
            return phi_potential(self.task, obs)
        except Exception:  # noqa: BLE001 - a physics gap is a shaping boundary
            return None

    def _budget(self):
        if self.budget is None:
            from ..transform.budget import ErrorBudget
            self.budget = ErrorBudget.for_op(getattr(self.task, "operation", ""), getattr(self.task, "dtype", "fp32"))
        return self.budget

    # ------------------------------------------------------------------ dispatch
    def call(self, name: str, args: Dict) -> Dict:
        v = validate_tool_call(name, args, self.schemas())
        if v["error"]:
            self.trace.append({"tool": name, "ok": False, "valid_name": v["valid_name"],
                               "valid_params": v["valid_params"], "error": v["error"]})
            return {"error": v["error"]}
        args = args or {}
        if name in EVAL_TOOLS:
            return self._evaluate(name, args.get("source") or self.current)
        if name == "revert":
            # right when the last evaluated kernel was not the best correct one
            last = next((t for t in reversed(self.trace) if t["tool"] in EVAL_TOOLS and "reward" in t), None)
            right = last is not None and (not last["ok"] or (self.best_reward is not None
                                                                and last["reward"] < self.best_reward))
            self.decisions.append({"action": "revert", "right": bool(right)})
            self.current = self.best or self.best_reward_src or self.current
            self.trace.append({"tool": name, "ok": True, "ms": self.best_ms, "valid_name": True,
                               "valid_params": True})
            return {"source": self.current}
        if name == "list_transforms":
            from ..transform.calculus import admissible_actions
            acts = admissible_actions(self.current, budget=self._budget())
            self.trace.append({"tool": name, "ok": True})
            return {"transforms": [{"name": a.name, "relation": a.kind, "epsilon": a.eps} for a in acts],
                    "budget_remaining": self._budget().remaining()}
        if name == "apply_transform":
            from ..transform.calculus import apply_sequence
            step = args.get("name", "")
            params = args.get("params") or {}
            from ..transform.library import get_transform
            t = get_transform(step)
            if t is None:
                self.trace.append({"tool": name, "ok": False})
                return {"applied": False, "reason": f"unknown transform {step!r}", "source": self.current}
            if params and hasattr(t, "actions"):
                from ..transform.calculus import Action
                t = Action(t, dict(params))
            new, applied, rejected, state = apply_sequence(self.current, [t], self._budget(), audit=True)
            ok = bool(applied)
            if ok:
                self.current = new
            self.trace.append({"tool": name, "ok": ok})
            out = {"applied": ok, "source": self.current, "budget_remaining": state["remaining"]}
            if not ok and rejected:
                out["reason"] = rejected[0].reason
            return out
        return {"error": f"unknown tool {name!r}"}

    def _evaluate(self, name: str, src: str) -> Dict:
        self.current = src
        obs = self.env.step(src)
        reward, correct, speedup = self._grade(obs, src)
        self.candidate_reward, self.candidate_correct = reward, correct
        self.candidate_speedup = None
        self.candidate_phi = None
        res: Dict = {"compiled": bool(obs.compiled), "correct": correct,
                     "snr_db": getattr(obs, "snr_by_shape", None) or getattr(obs, "snr_db", None)}
        if getattr(obs, "flagged_hack", False):
            res["rejected"] = obs.hack_reason
        if not obs.compiled:
            res["error"] = (getattr(obs, "error_text", "") or "")[-1500:]
        timed = name in ("bench", "keep", "pmc") and correct and obs.wall_ms
        if correct and (self.best_reward is None or reward > self.best_reward):
            self.best_reward, self.best_reward_src = reward, src
        if timed:
            res.update({"wall_ms": obs.wall_by_shape, "baseline_ms": obs.baseline_by_shape})
            if self.best_ms is None or obs.wall_ms < self.best_ms:
                self.best, self.best_ms = src, obs.wall_ms
            prev = self.best_speedup
            self.candidate_speedup = speedup
            self.candidate_phi = self._phi(obs)
            if speedup is not None:
                res["speedup"] = speedup
                res["best_speedup_so_far"] = max(prev or speedup, speedup)
                res["delta_vs_best"] = None if prev is None else speedup - prev
                res["improved_frontier"] = prev is None or speedup > prev
                if prev is None or speedup > prev:
                    self.best_speedup = speedup
        if name == "pmc" and correct:
            c = getattr(obs, "counters", None) or {}
            res["counters"] = c
            if c:
                from ..verifier.pmc import diagnose, top_stalls
                res["diagnosis"] = diagnose(c)
                res["top_stalls"] = top_stalls(c)
        if name == "keep":
            # right when the kept kernel is correct and at least as good as the best seen so far
            self.decisions.append({"action": "keep", "right": bool(correct and (self.best_reward is None
                                                                                or reward >= self.best_reward))})
            if correct:
                self.kept = src
        ent = {"tool": name, "ok": correct, "ms": obs.wall_ms, "reward": reward, "valid_name": True,
               "valid_params": True}
        if not correct:
            ent["error"] = ((getattr(obs, "error_text", "") or "") or
                            ("snr %s" % (getattr(obs, "snr_db", None),)))[-600:]
        self.trace.append(ent)
        return res

    def reseed(self) -> None:
        """Restart the working lineage from the seed (the best kernel and the
        frontier survive; the epsilon budget starts over)."""
        self.current = self.seed_src
        self.budget = None
        self.trace.append({"tool": "reseed", "ok": True})


_TOKEN = __import__("re").compile(r"[a-z0-9_]{4,}")


def _grounded(text: str, errors: List[str]) -> bool:
    """The text shares a word of four or more characters with an error the
    episode's tools reported."""
    words = set(_TOKEN.findall((text or "").lower()))
    return bool(words) and any(words & set(_TOKEN.findall(e.lower())) for e in errors)


def tool_use_breakdown(trace: List[Dict], final_correct: bool, *, reflections: Optional[List[str]] = None,
                       turns: int = 0, decisions: Optional[List[Dict]] = None) -> Dict[str, float]:
    """Components of the tool-use shaping reward, each in [0, 1] unless noted:

    * ``name`` / ``params``: fractions of calls naming a real tool with valid
      arguments;
    * ``order``: 1 when correctness was tested before the first bench;
    * ``commit``: 1 when a correct kernel was kept;
    * ``decisions``: mean of +1 (right) / -1 (wrong) keep and revert decisions,
      in [-1, 1];
    * ``reflection``: fraction of reflections that cite an error the tools
      reported (grounded), scaled by how many turns reflected;
    * ``failed``: fraction of evaluation calls that failed beyond the first
      two (a penalty).

    ``total`` = 0.03 name + 0.03 params + 0.05 order + 0.07 commit + 0.04
    decisions + 0.05 reflection - 0.1 failed, clipped to [-0.1, 0.25]: small
    against the verified kernel reward it is added to."""
    n = len(trace)
    if n == 0:
        return {"name": 0.0, "params": 0.0, "order": 0.0, "commit": 0.0, "decisions": 0.0, "reflection": 0.0,
                "failed": 0.0, "total": -0.1}
    names = [t["tool"] for t in trace]
    name_ok = sum(1 for t in trace if t.get("valid_name", True)) / n
    params_ok = sum(1 for t in trace if t.get("valid_params", True)) / n
    order = 1.0 if ("test" in names and "bench" in names and names.index("test") < names.index("bench")) else 0.0
    commit = 1.0 if ("keep" in names and final_correct) else 0.0
    ds = decisions or []
    dec = sum(1.0 if d.get("right") else -1.0 for d in ds) / len(ds) if ds else 0.0
    errors = [t["error"] for t in trace if t.get("error")]
    refl = 0.0
    if reflections:
        grounded = sum(1 for r in reflections if _grounded(r, errors) or not errors)
        refl = (grounded / len(reflections)) * min(1.0, len(reflections) / max(1, turns or len(reflections)))
    evals = [t for t in trace if t["tool"] in EVAL_TOOLS]
    fails = sum(1 for t in evals if not t.get("ok"))
    failed = max(0, fails - 2) / max(1, len(evals))
    total = (0.03 * name_ok + 0.03 * params_ok + 0.05 * order + 0.07 * commit + 0.04 * dec + 0.05 * refl
             - 0.1 * failed)
    return {"name": name_ok, "params": params_ok, "order": order, "commit": commit, "decisions": dec,
            "reflection": refl, "failed": failed, "total": max(-0.1, min(0.25, total))}


def tool_use_reward(trace: List[Dict], final_correct: bool, reflections=0, turns: int = 0,
                    decisions: Optional[List[Dict]] = None) -> float:
    """Total of :func:`tool_use_breakdown`; ``reflections`` is the list of the
    episode's reflection texts (an int count is accepted and treated as that
    many grounded reflections)."""
    if isinstance(reflections, int):
        refl = ["grounded"] * reflections
        trace = [dict(t, error=None) for t in trace]              # counts were already judged grounded
    else:
        refl = list(reflections or [])
    return tool_use_breakdown(trace, final_correct, reflections=refl, turns=turns, decisions=decisions)["total"]
