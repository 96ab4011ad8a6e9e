"""Transform calculus: typed, parameterised source-to-source rewrites of
kernel modules, the legal move set under an approximation budget, and
audited rewrite trajectories.

A :class:`Transformation` is a rewrite family: ``rewrite(src, **params)``
returns the new source or ``None`` when it does not apply; ``domain(src)``
lists the parameter choices that make sense for this source;
``side_conditions(src, params)`` returns the reasons a choice is illegal
(empty when legal); ``epsilon(params)`` is the tolerance an ``approx`` choice
spends. An :class:`Action` is one family with fixed parameters; it also
behaves like a parameterless transformation (``name``, ``kind``, ``eps``,
``apply(src)``), which is what the search and the agent tools enumerate.

``admissible_actions`` is the action space of the RL policy and of the
search: every (family, params) whose side conditions hold, whose epsilon
fits the remaining budget and that actually changes the source. Spending
budget only removes approximate actions, never adds any (monotone).
``apply_sequence`` runs a trajectory gating each step on (1) side
conditions, (2) budget, (3) applicability, and returns the new source with
an audit trail of what was applied, what was refused and why.

The typing is an action-space prior, not a proof; the environment's SNR
oracle verifies every rewritten kernel.
Reference behaviour: kore/transform/calculus.py:43-321.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple, Union

from .budget import APPROX, EXACT, ErrorBudget

Params = Dict[str, Any]


def _no_conditions(src: str, params: Params) -> List[str]:
    return []


@dataclass(frozen=True)
class Transformation:
    name: str
    kind: str                                               # "exact" | "approx"
    rewrite: Callable[..., Optional[str]]                   # rewrite(src, **params)
    eps: float = 0.0                                        # default epsilon (approx)
    knob: str = ""
    domain: Callable[[str], List[Params]] = lambda src: [{}]
    side_conditions: Callable[[str, Params], List[str]] = _no_conditions
    eps_fn: Optional[Callable[[Params], float]] = None
    doc: str = ""

    @property
    def relation(self) -> str:
        return self.kind

    def epsilon(self, params: Optional[Params] = None) -> float:
        if self.kind == EXACT:
            return 0.0
        return float(self.eps_fn(params or {})) if self.eps_fn is not None else float(self.eps)

    def apply(self, src: str, **params) -> Optional[str]:
        """The rewritten source, or None when illegal or a no-op."""
        if not params:
            dom = self.domain(src)
            params = dom[0] if dom else {}
        if self.side_conditions(src, params):
            return None
        try:
            out = self.rewrite(src, **params)
        except (ValueError, KeyError, IndexError):
            return None
        return out if out is not None and out != src else None

    def actions(self, src: str) -> List["Action"]:
        return [Action(self, dict(p)) for p in self.domain(src)]


@dataclass(frozen=True)
class Action:
    transform: Transformation
    params: Params = field(default_factory=dict)

    @property
    def name(self) -> str:
        if not self.params:
            return self.transform.name
        return self.transform.name + "(" + ",".join(f"{k}={v}" for k, v in sorted(self.params.items())) + ")"

    @property
    def kind(self) -> str:
        return self.transform.kind

    @property
    def eps(self) -> float:
        return self.transform.epsilon(self.params)

    def violations(self, src: str) -> List[str]:
        return self.transform.side_conditions(src, self.params)

    def apply(self, src: str) -> Optional[str]:
        if self.violations(src):
            return None
        try:
            out = self.transform.rewrite(src, **self.params)
        except (ValueError, KeyError, IndexError):
            return None
        return out if out is not None and out != src else None

    def as_step(self) -> Tuple[str, Params]:
        return self.transform.name, dict(self.params)

    def __hash__(self):
        return hash(self.name)


Step = Union[Action, Transformation, Tuple[str, Params], str]


@dataclass
class StepRecord:
    name: str
    relation: str
    eps: float
    reason: str = ""


def admissible_actions(src: str, library: Optional[Sequence[Transformation]] = None,
                       budget: Optional[ErrorBudget] = None) -> List[Action]:
    if library is None:
        from .library import LIBRARY
        library = LIBRARY
    budget = budget if budget is not None else ErrorBudget()
    out: List[Action] = []
    for t in library:
        for a in t.actions(src):
            if budget.affords(a.kind, a.eps) and a.apply(src) is not None:
                out.append(a)
    return out


def _resolve(step: Step, library: Sequence[Transformation]) -> Optional[Action]:
    if isinstance(step, Action):
        return step
    if isinstance(step, Transformation):
        return Action(step, {})
    if isinstance(step, str):
        step = (step, {})
    name, params = step
    for t in library:
        if t.name == name:
            return Action(t, dict(params or {}))
    return None


def apply_sequence(src: str, steps: Sequence[Step], budget: Optional[ErrorBudget] = None, *,
                   library: Optional[Sequence[Transformation]] = None, audit: bool = False):
    """Apply ``steps`` in order. Returns ``(src, applied_names)`` or, with
    ``audit=True``, ``(src, applied, rejected, budget_snapshot)`` where
    applied / rejected are :class:`StepRecord` lists."""
    if library is None:
        from .library import LIBRARY
        library = LIBRARY
    budget = budget if budget is not None else ErrorBudget()
    applied: List[StepRecord] = []
    rejected: List[StepRecord] = []
    for st in steps:
        a = _resolve(st, library)
        if a is None:
            rejected.append(StepRecord(str(st), "", 0.0, "unknown transform"))
            continue
        if not a.params:                     # a bare family: its first choice for this source
            dom = a.transform.domain(src)
            if dom and dom[0]:
                a = Action(a.transform, dict(dom[0]))
        why = a.violations(src)
        if why:
            rejected.append(StepRecord(a.name, a.kind, a.eps, "side condition: " + "; ".join(why)))
            continue
        if not budget.affords(a.kind, a.eps):
            rejected.append(StepRecord(a.name, a.kind, a.eps, f"budget: needs {a.eps}, {budget.remaining()} left"))
            continue
        out = a.apply(src)
        if out is None:
            rejected.append(StepRecord(a.name, a.kind, a.eps, "does not apply"))
            continue
        src = out
        budget.spend(a.name, a.kind, a.eps)
        applied.append(StepRecord(a.name, a.kind, a.eps))
    if audit:
        return src, applied, rejected, budget.snapshot()
    return src, [r.name for r in applied]


# ----------------------------------------------------------------------------- source helpers
def find_int_kwarg(src: str, name: str) -> Optional[int]:
    import re
    m = re.search(rf"\b{name}\s*=\s*(\d+)\b", src)
    return int(m.group(1)) if m else None


def set_int_kwarg(src: str, name: str, value: int) -> Optional[str]:
    """Replace the first ``name=<int>`` by ``name=value``."""
    import re
    m = re.search(rf"\b({name}\s*=\s*)(\d+)\b", src)
    if not m:
        return None
    return src[: m.start(2)] + str(int(value)) + src[m.end(2):]


def replace_int_kwarg(name: str, fn: Callable[[int], int]) -> Callable[..., Optional[str]]:
    def rw(src: str, **_) -> Optional[str]:
        v = find_int_kwarg(src, name)
        if v is None:
            return None
        new = fn(v)
        if new <= 0 or new == v:
            return None
        return set_int_kwarg(src, name, new)
    return rw


# older name kept for callers of the single-meter interface
EpsBudget = ErrorBudget
__all__ = ["Transformation", "Action", "StepRecord", "admissible_actions", "apply_sequence", "EpsBudget",
           "ErrorBudget", "EXACT", "APPROX", "find_int_kwarg", "set_int_kwarg", "replace_int_kwarg"]
