"""The production entry point of the search: the transform calculus as the
move generator, the verified environment as the grader.

``TransformProposePolicy`` turns a source into candidate edits (admissible
actions of the transform library, optionally extended with the discovered
families) with priors from a value model. A source without admissible moves
(e.g. a torch-reference seed) yields none, and the root comes back
unexpanded. ``search_from_kernel`` is what GRPO's rank-0 search-then-distill
hook calls: speedup samples against the task's vendor baseline from
``env.step``, LCB ranking, optional roofline branch-and-bound.

Reference behaviour: kore/search/propose.py:35-205.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Sequence

from ..transform.budget import ErrorBudget
from ..transform.calculus import Action, admissible_actions
from .alphakernel import CORRECT, COMPILE_FAIL, INCORRECT, INFRA, Eval, SearchResult, make_roofline_ub_fn, search


class TransformProposePolicy:
    """Move generator: admissible transform actions with value-model priors."""

    def __init__(self, value_fn: Optional[Callable[[str], float]] = None, *, discover: bool = False, library=None):
        self.value_fn = value_fn
        self.discover = discover
        self.library = library

    def library_for(self, src: str):
        if self.library is not None:
            return self.library
        if self.discover:
            from ..transform.discover import extend_library
            return extend_library(src, enabled=True)
        from ..transform.library import LIBRARY
        return LIBRARY

    def propose(self, src: str, budget: Optional[ErrorBudget] = None, k: int = 8) -> List[Action]:
        try:
            acts = admissible_actions(src, self.library_for(src), budget)
        except Exception:                     # an unparsable source proposes nothing
            return []
        if self.value_fn is not None:
            acts.sort(key=lambda a: self.value_fn(a.apply(src) or src), reverse=True)
        return acts[:k]

    def prior(self, src: str, action: str) -> float:
        if self.value_fn is None:
            return 1.0
        from ..transform.library import get_transform
        t = get_transform(action)
        child = t.apply(src) if t else None
        return self.value_fn(child) if child else 0.0


def model_value_fn(task=None, model=None) -> Callable[[str], float]:
    """A per-source prior from the value model (the trained default model when
    one is loaded, else its schedule heuristic), scored with the task's
    context and memoised per source."""
    from ..value.rerank import score_candidates
    cache: Dict[str, float] = {}

    def f(src: str) -> float:
        if src not in cache:
            cache[src] = float(score_candidates([src], task, model)[0])
        return cache[src]
    return f


def env_evaluator(env, baseline_ms: Optional[float] = None, ceiling=None) -> Callable[[str], Eval]:
    """Grade a source on the environment: status and one speedup sample."""
    def evaluate(s: str) -> Eval:
        obs = env.step(s)
        if getattr(obs, "infra_error", False):
            return Eval(INFRA)
        if not getattr(obs, "compiled", True):
            return Eval(COMPILE_FAIL)
        if not (obs.validation_passed and obs.wall_ms):
            return Eval(INCORRECT)
        base = obs.baseline_ms or baseline_ms
        if ceiling is not None:
            ceiling.observe_baseline(base)
        return Eval(CORRECT, base / obs.wall_ms if base else 1.0 / obs.wall_ms)
    return evaluate


def search_from_kernel(src: str, env, *, budget: int = 32, k_expand: int = 4, max_depth: int = 6,
                       bnb: bool = False, value_fn=None, baseline_ms: Optional[float] = None, task=None,
                       discover: bool = False, eps_budget: Optional[ErrorBudget] = None,
                       incumbent_min_measures: int = 1) -> SearchResult:
    """Search the rewrites of ``src`` with verified evaluations on ``env``;
    ``value_fn="model"`` takes the priors from the value model."""
    if value_fn == "model":
        value_fn = model_value_fn(task)
    ceiling = make_roofline_ub_fn(task) if (bnb and task is not None) else None
    pol = TransformProposePolicy(value_fn, discover=discover)
    if eps_budget is None and task is not None:
        eps_budget = ErrorBudget.for_op(task.operation, task.dtype)
    return search(src, env_evaluator(env, baseline_ms, ceiling), budget=budget, k_expand=k_expand,
                  max_depth=max_depth, prior_fn=pol.prior if value_fn else None, bnb=bnb and ceiling is not None,
                  ceiling_fn=ceiling, library=pol.library_for(src), eps_budget=eps_budget,
                  incumbent_min_measures=incumbent_min_measures)


def search_summary(res: SearchResult) -> Dict[str, object]:
    return {"best_speedup": res.best_score, "best_speedup_lcb": res.best_lcb, "path": res.path,
            "evaluated": res.evaluated, **res.stats}
