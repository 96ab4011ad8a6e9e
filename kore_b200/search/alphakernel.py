"""Best-first / PUCT search over transform sequences ("AlphaKernel").

Nodes are kernel sources; edges are admissible transforms. A node is
expanded with up to ``k_expand`` children ordered by the value-model prior;
children are verified (KoreEnv) and scored by speedup. Selection is PUCT
(mean + c * prior * sqrt(N_parent) / (1 + N)) or pure best-first by LCB.
With ``bnb`` a child whose roofline ceiling (T_min-based best possible
speedup) cannot beat the incumbent is pruned (branch-and-bound).
Reference parity: kore/search/alphakernel.py:382-959.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

from ..transform.calculus import EpsBudget
from ..transform.library import LIBRARY, admissible


@dataclass
class Node:
    src: str
    parent: Optional["Node"] = None
    action: str = ""
    depth: int = 0
    n: int = 0
    value: float = 0.0
    prior: float = 1.0
    score: Optional[float] = None           # measured speedup (None = not correct)
    children: List["Node"] = field(default_factory=list)
    expanded: bool = False


@dataclass
class SearchResult:
    best_src: str
    best_score: float
    evaluated: int
    path: List[str]


def search(root_src: str, evaluate: Callable[[str], Optional[float]], *, budget: int = 32, k_expand: int = 4,
           max_depth: int = 6, c_puct: float = 1.0, prior_fn: Optional[Callable[[str, str], float]] = None,
           ceiling_fn: Optional[Callable[[str], Optional[float]]] = None, bnb: bool = False,
           mode: str = "puct") -> SearchResult:
    root = Node(root_src, score=evaluate(root_src))
    best = root
    used = 1
    while used < budget:
        node = root
        while node.expanded and node.children:
            tot = math.sqrt(max(1, node.n))
            node = max(node.children, key=lambda ch: (ch.value / max(1, ch.n)) +
                       (c_puct * ch.prior * tot / (1 + ch.n) if mode == "puct" else 0.0))
        if node.depth >= max_depth or node.score is None:
            node.expanded = True
            if node is root and not root.children:
                break
            _backup(node, -1.0)
            if all(ch.expanded for ch in root.children) and used >= budget:
                break
            continue
        acts = admissible(node.src)
        if prior_fn is not None:
            acts.sort(key=lambda t: prior_fn(node.src, t.name), reverse=True)
        node.expanded = True
        made = 0
        for t in acts:
            if used >= budget or made >= k_expand:
                break
            child_src = t.apply(node.src)
            if child_src is None:
                continue
            if bnb and ceiling_fn is not None:
                ceil = ceiling_fn(child_src)
                if ceil is not None and best.score is not None and ceil <= best.score:
                    continue
            s = evaluate(child_src)
            used += 1
            made += 1
            ch = Node(child_src, node, t.name, node.depth + 1, prior=(prior_fn(node.src, t.name) if prior_fn else 1.0),
                      score=s)
            node.children.append(ch)
            _backup(ch, s if s is not None else -1.0)
            if s is not None and (best.score is None or s > best.score):
                best = ch
        if made == 0:
            _backup(node, node.score or -1.0)
            if node is root:
                break
    path, n = [], best
    while n.parent is not None:
        path.append(n.action)
        n = n.parent
    return SearchResult(best.src, best.score if best.score is not None else -1.0, used, list(reversed(path)))


def _backup(node: Node, v: float) -> None:
    while node is not None:
        node.n += 1
        node.value += v
        node = node.parent
