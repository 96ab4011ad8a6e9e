"""AlphaKernel: value-guided best-first search over kernel rewrites, with the
verified environment as an exact but expensive simulator.

State space: kernel sources. Moves: admissible actions of the transform
calculus (each node carries its own epsilon budget, so approximate moves run
out along a path). Every leaf is graded by the verifier: ``evaluate(src)``
returns a speedup sample (float), ``None`` for an incorrect kernel, or an
:class:`Eval` with an explicit status.

* Nodes are de-duplicated by a fingerprint of the canonicalised source (a
  transposition table): a kernel reached by a second path is linked into the
  DAG and inherits its measurements, with no new verifier call.
* Selection is PUCT over the whole frontier: backed-up value + prior x
  sqrt(total visits) / (1 + visits) + a novelty bonus for shallow nodes.
  Incorrect nodes stay in the frontier with a low value (a later rewrite can
  repair them, e.g. a mask).
* Backup is MAX: a node's value is the best LCB in its sub-DAG, so the search
  commits to the single best kernel it can reach rather than an average.
* Measurements are allocated by successive halving: every correct kernel gets
  one sample, the better half of the candidates get more (up to
  ``sh_max_measures``), and kernels are ranked by the LCB of their speedup.
* Branch-and-bound: with a ceiling function (the best speedup any kernel for
  the task can reach, e.g. baseline time / roofline time) a node whose
  ceiling is not above the pruning floor is never evaluated or expanded. The
  floor is the running max of achieved LCBs, kept separate from the reported
  incumbent (an LCB can drop when re-measured; a pruning decision must not be
  revisited).
* The incumbent is recomputed as the argmax over correct nodes with at least
  ``incumbent_min_measures`` samples.

Reference behaviour: kore/search/alphakernel.py:382-959.
"""
from __future__ import annotations

import hashlib
import math
import re
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Union

from ..transform.budget import ErrorBudget
from ..transform.calculus import Action, admissible_actions
from .bandit import Budget, MeasureStats

CORRECT, INCORRECT, COMPILE_FAIL, INFRA, PRUNED = "correct", "incorrect", "compile_fail", "infra", "pruned"


@dataclass
class Eval:
    status: str
    speedup: Optional[float] = None


def fingerprint(src: str) -> str:
    """Hash of the source with comments, blank lines and spacing removed."""
    lines = []
    for line in src.splitlines():
        line = re.sub(r"#.*$", "", line).rstrip()
        if line.strip():
            lines.append(re.sub(r"[ \t]+", " ", line))
    return hashlib.sha1("\n".join(lines).encode()).hexdigest()[:20]


@dataclass
class Node:
    src: str
    fp: str
    depth: int = 0
    parent: Optional["Node"] = None             # first discovery (the reported path)
    action: str = ""
    parents: List["Node"] = field(default_factory=list)
    children: List["Node"] = field(default_factory=list)
    status: str = "pending"
    stats: MeasureStats = field(default_factory=MeasureStats)
    prior: float = 1.0
    ceiling: Optional[float] = None
    best: float = -math.inf                     # MAX-backed-up value of the sub-DAG
    visits: int = 0
    expanded: bool = False
    eps: Optional[ErrorBudget] = None

    # compatibility with the earlier node record
    @property
    def n(self) -> int:
        return self.visits

    @property
    def score(self) -> Optional[float]:
        return self.stats.mean if self.status == CORRECT and self.stats.n else None

    def value(self, z: float) -> float:
        if self.status == CORRECT and self.stats.n:
            return self.stats.lcb(z)
        return -1.0


@dataclass
class SearchResult:
    best_src: str
    best_score: float
    evaluated: int
    path: List[str]
    best_lcb: float = -math.inf
    stats: Dict[str, int] = field(default_factory=dict)


Evaluator = Callable[[str], Union[None, float, Eval]]


class AlphaKernel:
    """One search over the rewrites of a root kernel (see module docstring)."""

    def __init__(self, evaluate: Evaluator, *, budget: int = 32, k_expand: int = 4, max_depth: Optional[int] = 6,
                 c_puct: float = 1.0, z: float = 1.0, prior_fn: Optional[Callable[[str, str], float]] = None,
                 value_fn: Optional[Callable[[Sequence[str]], Sequence[float]]] = None,
                 ceiling_fn: Optional[Callable[[str], Optional[float]]] = None, bnb: bool = False,
                 mode: str = "puct", sh_max_measures: int = 4, incumbent_min_measures: int = 1,
                 novelty: float = 0.05, library=None, eps_budget: Optional[ErrorBudget] = None):
        self.evaluate_fn = evaluate
        self.budget = Budget(budget)
        self.k_expand, self.max_depth = k_expand, max_depth
        self.c_puct, self.z, self.mode = c_puct, z, mode
        self.prior_fn, self.value_fn, self.ceiling_fn = prior_fn, value_fn, ceiling_fn
        self.bnb = bnb
        self.sh_max, self.inc_min = sh_max_measures, incumbent_min_measures
        self.novelty = novelty
        self.library = library
        self.eps0 = eps_budget if eps_budget is not None else ErrorBudget(total=0.05)
        self.table: Dict[str, Node] = {}
        self.nodes: List[Node] = []
        self.incumbent: Optional[Node] = None
        self.prune_floor = -math.inf
        self.counters = {"evaluated": 0, "linked": 0, "pruned": 0, "expanded": 0, "remeasured": 0}

    # ------------------------------------------------------------------ grading
    def _grade(self, node: Node) -> None:
        if not self.budget.take():
            return
        self.counters["evaluated"] += 1
        r = self.evaluate_fn(node.src)
        if isinstance(r, Eval):
            node.status = r.status
            if r.status == CORRECT and r.speedup is not None:
                node.stats.add(float(r.speedup))
        elif r is None:
            node.status = INCORRECT
        else:
            node.status = CORRECT
            node.stats.add(float(r))

    def _remeasure(self, node: Node) -> bool:
        if not self.budget.take():
            return False
        self.counters["evaluated"] += 1
        self.counters["remeasured"] += 1
        r = self.evaluate_fn(node.src)
        s = r.speedup if isinstance(r, Eval) else r
        if s is not None:
            node.stats.add(float(s))
        return True

    # ------------------------------------------------------------------ bookkeeping
    def _backup(self, node: Node) -> None:
        """MAX backup of the node's value through every parent in the DAG."""
        stack, seen = [node], set()
        node.best = max(node.best, node.value(self.z))
        while stack:
            n = stack.pop()
            if id(n) in seen:
                continue
            seen.add(id(n))
            n.visits += 1
            for p in n.parents:
                if n.best > p.best:
                    p.best = n.best
                stack.append(p)

    def _update_incumbent(self) -> None:
        ok = [n for n in self.nodes if n.status == CORRECT and n.stats.n >= self.inc_min]
        if not ok:
            ok = [n for n in self.nodes if n.status == CORRECT and n.stats.n]
        if ok:
            self.incumbent = max(ok, key=lambda n: (n.stats.lcb(self.z), n.stats.mean))
            self.prune_floor = max(self.prune_floor, self.incumbent.stats.lcb(self.z))

    def _dominated(self, node: Node) -> bool:
        return (self.bnb and node.ceiling is not None and self.incumbent is not None
                and node.ceiling <= self.prune_floor)

    def _refine(self) -> None:
        """Successive-halving step: one more sample for the better half of the
        correct candidates that still have fewer than ``sh_max`` samples."""
        cand = [n for n in self.nodes if n.status == CORRECT and 0 < n.stats.n < self.sh_max]
        if len(cand) < 1:
            return
        cand.sort(key=lambda n: (n.stats.lcb(self.z), n.stats.mean), reverse=True)
        for n in cand[: max(1, len(cand) // 2)]:
            if not self._remeasure(n):
                break
            self._backup(n)

    # ------------------------------------------------------------------ tree ops
    def _node(self, src: str, parent: Optional[Node], action: str, prior: float) -> Optional[Node]:
        fp = fingerprint(src)
        if fp in self.table:                           # transposition: link, no new grading
            old = self.table[fp]
            if parent is not None and parent not in old.parents and old is not parent:
                old.parents.append(parent)
                parent.children.append(old)
                self.counters["linked"] += 1
                self._backup(old)
            return None
        depth = parent.depth + 1 if parent else 0
        n = Node(src, fp, depth, parent, action, [parent] if parent else [], prior=prior)
        n.eps = (parent.eps.copy() if parent and parent.eps else self.eps0.copy())
        if self.ceiling_fn is not None:
            n.ceiling = self.ceiling_fn(src)
        self.table[fp] = n
        self.nodes.append(n)
        if parent is not None:
            parent.children.append(n)
        return n

    def _select(self) -> Optional[Node]:
        frontier = [n for n in self.nodes if not n.expanded and n.status in (CORRECT, INCORRECT)
                    and (self.max_depth is None or n.depth < self.max_depth)]
        live = []
        for n in frontier:
            if self._dominated(n):
                n.expanded = True
                n.status = PRUNED if n.status != CORRECT else n.status
                self.counters["pruned"] += 1
            else:
                live.append(n)
        if not live:
            return None
        total = math.sqrt(max(1, sum(n.visits for n in self.nodes)))

        def acq(n: Node) -> float:
            v = n.best if n.best > -math.inf else n.value(self.z)
            if self.mode != "puct":
                return v
            return v + self.c_puct * n.prior * total / (1 + n.visits) + self.novelty / (1 + n.depth)
        return max(live, key=acq)

    def _expand(self, node: Node) -> int:
        node.expanded = True
        self.counters["expanded"] += 1
        acts: List[Action] = admissible_actions(node.src, self.library, node.eps)
        if not acts:
            return 0
        priors = [1.0] * len(acts)
        if self.value_fn is not None:
            kids = [a.apply(node.src) or node.src for a in acts]
            priors = list(self.value_fn(kids))
        elif self.prior_fn is not None:
            priors = [self.prior_fn(node.src, a.name) for a in acts]
        order = sorted(range(len(acts)), key=lambda i: priors[i], reverse=True)
        s = sum(max(p, 0.0) for p in priors) or 1.0
        made = 0
        for i in order:
            if made >= self.k_expand or self.budget.exhausted():
                break
            a = acts[i]
            child_src = a.apply(node.src)
            if child_src is None:
                continue
            ch = self._node(child_src, node, a.name, max(priors[i], 0.0) / s * len(acts))
            if ch is None:
                continue
            ch.eps.spend(a.name, a.kind, a.eps)
            if self._dominated(ch):
                ch.status, ch.expanded = PRUNED, True
                self.counters["pruned"] += 1
                continue
            self._grade(ch)
            made += 1
            self._backup(ch)
            self._update_incumbent()
        return made

    # ------------------------------------------------------------------ run
    def run(self, root_src: str) -> SearchResult:
        root = self._node(root_src, None, "", 1.0)
        self._grade(root)
        self._backup(root)
        self._update_incumbent()
        while not self.budget.exhausted():
            node = self._select()
            if node is None:
                self._refine()
                if not any(n.status == CORRECT and n.stats.n < self.sh_max for n in self.nodes):
                    break
                continue
            self._expand(node)
            self._refine()
            self._update_incumbent()
        best = self.incumbent or root
        path, n = [], best
        while n.parent is not None:
            path.append(n.action)
            n = n.parent
        score = best.stats.mean if best.status == CORRECT and best.stats.n else -1.0
        return SearchResult(best.src, score, self.counters["evaluated"], list(reversed(path)),
                            best.stats.lcb(self.z) if best.stats.n else -math.inf,
                            dict(self.counters, nodes=len(self.nodes)))


def search(root_src: str, evaluate: Evaluator, *, budget: int = 32, k_expand: int = 4, max_depth: Optional[int] = 6,
           c_puct: float = 1.0, prior_fn=None, ceiling_fn=None, bnb: bool = False, mode: str = "puct",
           **kw) -> SearchResult:
    return AlphaKernel(evaluate, budget=budget, k_expand=k_expand, max_depth=max_depth, c_puct=c_puct,
                       prior_fn=prior_fn, ceiling_fn=ceiling_fn, bnb=bnb, mode=mode, **kw).run(root_src)


class RooflineCeiling:
    """Admissible ceiling of a task: baseline time / roofline time. The
    baseline is learned from the environment's observations
    (``observe_baseline``); until then there is no ceiling (no pruning).
    ``safety_margin`` leaves headroom for precision-lowering moves."""

    def __init__(self, t_min_ms: float, baseline_ms: Optional[float] = None, safety_margin: float = 0.25):
        self.t_min_ms, self.baseline_ms, self.margin = float(t_min_ms), baseline_ms, safety_margin

    def observe_baseline(self, ms: Optional[float]) -> None:
        if ms and ms > 0:
            self.baseline_ms = ms if self.baseline_ms is None else min(self.baseline_ms, ms)

    def __call__(self, src: str = "", task=None) -> Optional[float]:
        if not self.baseline_ms or self.t_min_ms <= 0:
            return None
        return self.baseline_ms / self.t_min_ms * (1.0 + self.margin)


def make_roofline_ub_fn(task, dtype: Optional[str] = None, safety_margin: float = 0.25) -> Optional[RooflineCeiling]:
    """A :class:`RooflineCeiling` from the task's primary shape (None when the
    operation has no roofline model)."""
    from ..analysis.rooflines import detect_arch, resolve_peaks, roofline
    shape = task.shapes[-1] if getattr(task, "shapes", None) else None
    if shape is None:
        return None
    arch = detect_arch()
    r = roofline(task.task_id, task.operation, dtype or task.dtype, shape.name, shape.dims,
                 resolve_peaks(arch), arch)
    if r is None or not getattr(r, "t_min_ms", None):
        return None
    return RooflineCeiling(r.t_min_ms, safety_margin=safety_margin)
