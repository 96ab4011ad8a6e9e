"""Approximation budget of a rewrite trajectory and the relation lattice.

Every rewrite is typed by how its output relates to its input:

* ``exact``  - bit-preserving (scheduling, pipelining, occupancy, masks that
  guard accesses the kernel already makes, hints the compiler may ignore);
* ``approx`` - equal within a tolerance epsilon (anything that can reorder a
  floating-point reduction, change a precision or a tile shape of a reduction).

Relations form a two-point lattice with ``exact`` as its bottom: composing
any ``approx`` step into a trajectory makes it ``approx`` and the trajectory's
contract is its loosest step (max epsilon). Independently the budget meters
the *sum* of epsilons spent, which is what admits or refuses the next
approximate step; the two answer different questions (what the result is
guaranteed to be vs. how much drift the search may still buy).

The default budget of a task is the tolerance of its dtype scaled by how
error-amplifying its operation is (deep reductions get less, elementwise
maps more). Downstream, the environment's SNR gate remains the authority on
correctness; the budget only bounds what the search may try.

Reference behaviour: kore/transform/budget.py:1-289 (lattice, per-(op,dtype)
defaults, spend/remaining).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Tuple

EXACT = "exact"
APPROX = "approx"
RELATIONS = (EXACT, APPROX)

# tolerance a dtype's verification already grants (relative error scale)
DTYPE_EPS: Dict[str, float] = {
    "fp64": 0.005, "fp32": 0.02, "tf32": 0.04, "fp16": 0.08, "bf16": 0.10,
    "fp8": 0.25, "fp8_e4m3": 0.25, "fp8_e5m2": 0.30, "int8": 0.15, "mxfp4": 0.35, "fp4": 0.35,
}

# how much an operation amplifies per-step perturbations (multiplier on DTYPE_EPS)
OP_SCALE: Tuple[Tuple[str, float], ...] = (
    ("attention", 0.5), ("flash", 0.5), ("gemm", 0.6), ("matmul", 0.6), ("conv", 0.6), ("bmm", 0.6),
    ("moe", 0.6), ("scan", 0.5), ("ssm", 0.5), ("cumsum", 0.5), ("softmax", 0.8), ("norm", 0.8),
    ("reduce", 0.7), ("sum", 0.7), ("loss", 0.7), ("entropy", 0.7), ("quant", 0.9),
    ("elementwise", 1.5), ("activation", 1.5), ("gelu", 1.5), ("silu", 1.5), ("relu", 1.5),
    ("add", 1.5), ("mul", 1.5), ("copy", 1.5), ("transpose", 1.5),
)


def op_scale(operation: str) -> float:
    op = (operation or "").lower()
    for key, s in OP_SCALE:
        if key in op:
            return s
    return 1.0


def default_epsilon(operation: str, dtype: str) -> float:
    return DTYPE_EPS.get((dtype or "fp32").lower(), 0.05) * op_scale(operation)


def compose_relation(a: str, b: str) -> str:
    """Lattice join: exact only if both are exact."""
    if a not in RELATIONS or b not in RELATIONS:
        raise ValueError(f"unknown relation {a!r} / {b!r}")
    return EXACT if a == EXACT and b == EXACT else APPROX


def compose_eps(a: float, b: float) -> float:
    """Contract tolerance of two composed steps: the looser one."""
    return max(float(a), float(b))


def compose_all(steps: Iterable[Tuple[str, float]]) -> Tuple[str, float]:
    rel, eps = EXACT, 0.0
    for r, e in steps:
        rel = compose_relation(rel, r)
        eps = compose_eps(eps, e if r == APPROX else 0.0)
    return rel, eps


@dataclass
class ErrorBudget:
    """Additive epsilon meter plus the composed contract of what was applied."""

    total: float = 0.05
    spent: float = 0.0
    history: List[Tuple[str, str, float]] = field(default_factory=list)   # (name, relation, eps)

    @classmethod
    def for_op(cls, operation: str, dtype: str, scale: float = 1.0) -> "ErrorBudget":
        return cls(total=default_epsilon(operation, dtype) * scale)

    def remaining(self) -> float:
        return max(0.0, self.total - self.spent)

    def affords(self, relation: str, eps: float) -> bool:
        return relation == EXACT or self.spent + float(eps) <= self.total + 1e-12

    def spend(self, name: str, relation: str, eps: float) -> None:
        if not self.affords(relation, eps):
            raise ValueError(f"{name}: epsilon {eps} exceeds the remaining budget {self.remaining()}")
        if relation == APPROX:
            self.spent += float(eps)
        self.history.append((name, relation, float(eps) if relation == APPROX else 0.0))

    def composed_relation(self) -> str:
        return compose_all((r, e) for _, r, e in self.history)[0]

    def weakest_eps(self) -> float:
        return compose_all((r, e) for _, r, e in self.history)[1]

    def copy(self) -> "ErrorBudget":
        return ErrorBudget(self.total, self.spent, list(self.history))

    def snapshot(self) -> Dict[str, object]:
        return {"total": self.total, "spent": round(self.spent, 9), "remaining": round(self.remaining(), 9),
                "relation": self.composed_relation(), "weakest_eps": self.weakest_eps(),
                "steps": [h[0] for h in self.history]}

    # compatibility with the older single-meter interface
    @staticmethod
    def _eps_of(t) -> float:
        return t.epsilon() if hasattr(t, "epsilon") else getattr(t, "eps", 0.0)

    def can_afford(self, t) -> bool:
        return self.affords(getattr(t, "kind", EXACT), self._eps_of(t))

    def charge(self, t) -> None:
        self.spend(t.name, getattr(t, "kind", EXACT), self._eps_of(t))


def budget_from(value: Optional[object], operation: str = "", dtype: str = "fp32") -> ErrorBudget:
    if isinstance(value, ErrorBudget):
        return value
    if value is None:
        return ErrorBudget.for_op(operation, dtype)
    return ErrorBudget(total=float(value))
