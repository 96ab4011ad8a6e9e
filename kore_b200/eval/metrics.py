"""Kernel-evaluation metrics and paired statistics.

* ``fast_p(results, p)``: fraction of tasks whose candidate is correct AND
  at least p times faster than the baseline (KernelBench's fast_p).
* paired bootstrap CI of the mean difference, the exact two-sided sign
  test, and the Wilcoxon signed-rank test (normal approximation with tie
  and zero handling).
Reference parity: kore/eval/fastp.py:42, paired_stats.py.
"""
from __future__ import annotations

import math
import random
from typing import Dict, Iterable, List, Optional, Sequence, Tuple


def fast_p(results: Iterable[Dict], p: float = 1.0) -> float:
    rs = list(results)
    if not rs:
        return 0.0
    good = sum(1 for r in rs if r.get("correct") and (r.get("speedup") or 0.0) >= p)
    return good / len(rs)


def bootstrap_ci(a: Sequence[float], b: Sequence[float], iters: int = 2000, alpha: float = 0.05,
                 seed: int = 0) -> Tuple[float, float, float]:
    d = [x - y for x, y in zip(a, b)]
    n = len(d)
    if n == 0:
        return 0.0, 0.0, 0.0
    rng = random.Random(seed)
    means = sorted(sum(d[rng.randrange(n)] for _ in range(n)) / n for _ in range(iters))
    return sum(d) / n, means[int(alpha / 2 * iters)], means[int((1 - alpha / 2) * iters) - 1]


def sign_test(a: Sequence[float], b: Sequence[float]) -> float:
    """Exact two-sided binomial p-value on the signs of a - b (ties dropped)."""
    pos = sum(1 for x, y in zip(a, b) if x > y)
    neg = sum(1 for x, y in zip(a, b) if x < y)
    n = pos + neg
    if n == 0:
        return 1.0
    k = min(pos, neg)
    tail = sum(math.comb(n, i) for i in range(k + 1)) / 2 ** n
    return min(1.0, 2 * tail)


def wilcoxon(a: Sequence[float], b: Sequence[float]) -> float:
    """Two-sided p-value of the Wilcoxon signed-rank test (normal approximation)."""
    d = [x - y for x, y in zip(a, b) if x != y]
    n = len(d)
    if n == 0:
        return 1.0
    order = sorted(range(n), key=lambda i: abs(d[i]))
    ranks = [0.0] * n
    i = 0
    while i < n:
        j = i
        while j + 1 < n and abs(d[order[j + 1]]) == abs(d[order[i]]):
            j += 1
        for k in range(i, j + 1):
            ranks[order[k]] = (i + j) / 2 + 1
        i = j + 1
    w = sum(r for r, x in zip(ranks, d) if x > 0)
    mu = n * (n + 1) / 4
    sd = math.sqrt(n * (n + 1) * (2 * n + 1) / 24)
    z = (w - mu) / sd if sd else 0.0
    return math.erfc(abs(z) / math.sqrt(2))
