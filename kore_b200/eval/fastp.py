"""fast_p and its best-of-N relatives, with timing-integrity gating.

    fast_p = #{tasks correct AND baseline / time > p} / n

with ``n`` the full split (unattempted or failed tasks count as 0). The
speedup that enters it is gated first (:func:`gated_speedup`): a ratio above
``max_ratio`` is treated as a measurement artifact and capped, and a
measurement whose coefficient of variation exceeds ``max_cv_pct`` is damped
to at most 1x, so a glitch or a noisy bench cannot farm the metric.

* ``pass_at_k(n, c, k)``  unbiased estimator 1 - C(n-c, k) / C(n, k) of the
  probability that at least one of k samples (of n drawn, c correct) passes;
* ``fast_p_at_k(samples, p, k)``  the same estimator with "correct and faster
  than p" as success, averaged over tasks;
* ``fast_p_curve``  fast_p over a grid of p;
* ``multi_seed``  mean and a t-based confidence interval over seeds.

Reference behaviour: kore/eval/fastp.py (metric, pass@k, fast_p@k, multi-seed
intervals, timing-integrity gating).
"""
from __future__ import annotations

import math
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

P_GRID = (0.0, 0.5, 1.0, 1.5, 2.0)


def gated_speedup(speedup: Optional[float], cv_pct: Optional[float] = None, *, max_ratio: float = 50.0,
                  max_cv_pct: float = 5.0) -> float:
    if speedup is None or not math.isfinite(speedup) or speedup <= 0:
        return 0.0
    s = min(float(speedup), max_ratio)
    if cv_pct is not None and cv_pct > max_cv_pct:
        s = min(s, 1.0)
    return s


def _ok(r: Dict, p: float) -> bool:
    return bool(r.get("correct")) and gated_speedup(r.get("speedup"), r.get("cv_pct")) > p


def fast_p(results: Iterable[Dict], p: float = 1.0, n: Optional[int] = None) -> float:
    rs = list(results)
    denom = n if n is not None else len(rs)
    return sum(1 for r in rs if _ok(r, p)) / denom if denom else 0.0


def fast_p_curve(results: Sequence[Dict], grid: Sequence[float] = P_GRID, n: Optional[int] = None) -> Dict[str, float]:
    return {f"fast_{p}": fast_p(results, p, n) for p in grid}


def pass_at_k(n: int, c: int, k: int) -> float:
    """Unbiased pass@k from n samples with c successes."""
    if n <= 0 or k <= 0:
        return 0.0
    if n - c < k:
        return 1.0
    prod = 1.0
    for i in range(n - c + 1, n + 1):       # C(n-c, k) / C(n, k) as a product
        prod *= 1.0 - k / i
    return 1.0 - prod


def fast_p_at_k(samples: Dict[str, Sequence[Dict]], p: float = 1.0, k: int = 1) -> float:
    """``samples``: task -> list of sampled results (each {correct, speedup})."""
    if not samples:
        return 0.0
    vals = []
    for rs in samples.values():
        rs = list(rs)
        vals.append(pass_at_k(len(rs), sum(1 for r in rs if _ok(r, p)), k))
    return sum(vals) / len(vals)


_T975 = {1: 12.706, 2: 4.303, 3: 3.182, 4: 2.776, 5: 2.571, 6: 2.447, 7: 2.365, 8: 2.306, 9: 2.262, 10: 2.228,
         15: 2.131, 20: 2.086, 30: 2.042}


def _t975(df: int) -> float:
    if df in _T975:
        return _T975[df]
    keys = sorted(_T975)
    for a, b in zip(keys, keys[1:]):
        if a < df < b:
            return _T975[a] + (_T975[b] - _T975[a]) * (df - a) / (b - a)
    return 1.96


def multi_seed(values: Sequence[float]) -> Tuple[float, float, float]:
    """(mean, low, high) of a 95% t interval over per-seed values."""
    v = [float(x) for x in values]
    n = len(v)
    if n == 0:
        return 0.0, 0.0, 0.0
    m = sum(v) / n
    if n == 1:
        return m, m, m
    sd = math.sqrt(sum((x - m) ** 2 for x in v) / (n - 1))
    h = _t975(n - 1) * sd / math.sqrt(n)
    return m, m - h, m + h


def multi_seed_fast_p(runs: Sequence[Sequence[Dict]], p: float = 1.0, n: Optional[int] = None) -> Dict[str, float]:
    m, lo, hi = multi_seed([fast_p(r, p, n) for r in runs])
    return {"mean": m, "ci_low": lo, "ci_high": hi, "seeds": len(runs)}
