"""Transform calculus: typed source-to-source rewrites of kernel modules.

A :class:`Transformation` is *exact* (semantics-preserving: re-tiling,
warp count, pipeline depth, load vectorisation) or *approximate* with an
error budget epsilon (fast-math exponentials, reduced-precision
accumulation). ``apply_sequence`` composes transforms, skipping those whose
precondition fails, and tracks the spent approximation budget;
``admissible_actions`` lists what applies to a source under a remaining
budget. Reference parity: kore/transform/calculus.py:43-321, budget.py:185.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple


@dataclass(frozen=True)
class Transformation:
    name: str
    kind: str                                  # "exact" | "approx"
    rewrite: Callable[[str], Optional[str]]
    eps: float = 0.0                           # approximation budget consumed
    precondition: Callable[[str], bool] = lambda s: True
    doc: str = ""

    def apply(self, src: str) -> Optional[str]:
        if not self.precondition(src):
            return None
        out = self.rewrite(src)
        return out if out is not None and out != src else None


@dataclass
class EpsBudget:
    total: float = 0.05
    spent: float = 0.0
    history: List[str] = field(default_factory=list)

    def can_afford(self, t: Transformation) -> bool:
        return t.kind == "exact" or self.spent + t.eps <= self.total + 1e-12

    def charge(self, t: Transformation) -> None:
        if t.kind == "approx":
            self.spent += t.eps
        self.history.append(t.name)


def apply_sequence(src: str, seq: Sequence[Transformation], budget: Optional[EpsBudget] = None
                   ) -> Tuple[str, List[str]]:
    applied = []
    budget = budget or EpsBudget()
    for t in seq:
        if not budget.can_afford(t):
            continue
        out = t.apply(src)
        if out is not None:
            src = out
            budget.charge(t)
            applied.append(t.name)
    return src, applied


def admissible_actions(src: str, library: Sequence[Transformation], budget: Optional[EpsBudget] = None
                       ) -> List[Transformation]:
    budget = budget or EpsBudget()
    return [t for t in library if budget.can_afford(t) and t.apply(src) is not None]


def replace_int_kwarg(name: str, fn: Callable[[int], int]) -> Callable[[str], Optional[str]]:
    pat = re.compile(rf"\b({name}\s*=\s*)(\d+)")

    def rw(src: str) -> Optional[str]:
        m = pat.search(src)
        if not m:
            return None
        new = fn(int(m.group(2)))
        if new <= 0 or new == int(m.group(2)):
            return None
        return src[: m.start(2)] + str(new) + src[m.end(2):]
    return rw
