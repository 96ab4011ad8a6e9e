"""Search entry points used by GRPO's periodic search-then-distill hook
(reference parity: kore/search/propose.py:35-205)."""
from __future__ import annotations

from typing import Callable, Optional

from .alphakernel import SearchResult, search


class TransformProposePolicy:
    """Prior over transforms from a value model (or uniform)."""

    def __init__(self, value_fn: Optional[Callable[[str], float]] = None):
        self.value_fn = value_fn

    def prior(self, src: str, action: str) -> float:
        if self.value_fn is None:
            return 1.0
        from ..transform.library import get_transform
        t = get_transform(action)
        child = t.apply(src) if t else None
        return self.value_fn(child) if child else 0.0


def search_from_kernel(src: str, env, *, budget: int = 32, k_expand: int = 4, max_depth: int = 6,
                       bnb: bool = False, value_fn=None, baseline_ms: Optional[float] = None) -> SearchResult:
    """Search transforms of ``src`` with verified evaluations on ``env`` (speedup
    vs the vendor baseline; None for incorrect)."""
    def evaluate(s: str):
        obs = env.step(s)
        if not (obs.validation_passed and obs.wall_ms):
            return None
        base = obs.baseline_ms or baseline_ms
        return base / obs.wall_ms if base else 1.0 / obs.wall_ms

    pol = TransformProposePolicy(value_fn)
    return search(src, evaluate, budget=budget, k_expand=k_expand, max_depth=max_depth,
                  prior_fn=pol.prior if value_fn else None, bnb=bnb)
