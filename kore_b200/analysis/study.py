"""Speed-of-light study: does the roofline attainment eta = T_min / T_measured
explain measured speedups, and does a counter-based residual decomposition
explain measured time?

Three checks, each with a percentile-bootstrap 95% confidence interval:

(a) Spearman rank correlation between eta and speedup-vs-vendor over
    (task, candidate) records;
(b) R^2 of the ordinary least-squares residual model
    T_measured ~ T_min + b1 * stall_ms + b2 * occupancy_deficit_ms;
(c) monotone-in-valley: over pairs of candidates of the same task whose eta
    differ by at least ``gap``, the fraction where the higher-eta one is faster.

``leave_one_family_out`` fits (b) on all families but one and reports the R^2
on the held-out family (transfer of the residual model).
``bottleneck_from_counters`` names the limiter of one kernel from ncu
counters: tensor pipe, DRAM, latency / occupancy, or launch.
Reference parity: kore/analysis/p0_sol.py:449-597, residual_transfer.py:117,
analysis/roofline.py:98-507 (bottleneck_from_counters, attained_fraction).
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np


@dataclass
class Record:
    task_id: str
    family: str
    eta: float
    speedup: float
    t_measured_ms: float
    t_min_ms: float
    stall_ms: float = 0.0
    occ_deficit_ms: float = 0.0


def _rank(x: Sequence[float]) -> np.ndarray:
    x = np.asarray(x, dtype=float)
    order = np.argsort(x, kind="mergesort")
    r = np.empty(len(x))
    i = 0
    while i < len(x):
        j = i
        while j + 1 < len(x) and x[order[j + 1]] == x[order[i]]:
            j += 1
        r[order[i:j + 1]] = (i + j) / 2.0
        i = j + 1
    return r


def spearman(x: Sequence[float], y: Sequence[float]) -> float:
    if len(x) < 3:
        return float("nan")
    a, b = _rank(x), _rank(y)
    a, b = a - a.mean(), b - b.mean()
    den = math.sqrt(float((a * a).sum() * (b * b).sum()))
    return float((a * b).sum() / den) if den else float("nan")


def ols_r2(X: np.ndarray, y: np.ndarray) -> Tuple[np.ndarray, float]:
    coef, *_ = np.linalg.lstsq(X, y, rcond=None)
    res = y - X @ coef
    tot = ((y - y.mean()) ** 2).sum()
    return coef, float(1 - (res ** 2).sum() / tot) if tot > 0 else float("nan")


def _design(rs: Sequence[Record]) -> Tuple[np.ndarray, np.ndarray]:
    X = np.array([[r.t_min_ms, r.stall_ms, r.occ_deficit_ms, 1.0] for r in rs])
    y = np.array([r.t_measured_ms for r in rs])
    return X, y


def residual_r2(rs: Sequence[Record]) -> float:
    X, y = _design(rs)
    return ols_r2(X, y)[1]


def monotone_fraction(rs: Sequence[Record], gap: float = 0.05) -> float:
    by: Dict[str, List[Record]] = {}
    for r in rs:
        by.setdefault(r.task_id, []).append(r)
    good = tot = 0
    for group in by.values():
        for i in range(len(group)):
            for j in range(i + 1, len(group)):
                a, b = group[i], group[j]
                if abs(a.eta - b.eta) < gap:
                    continue
                hi, lo = (a, b) if a.eta > b.eta else (b, a)
                tot += 1
                good += hi.t_measured_ms < lo.t_measured_ms
    return good / tot if tot else float("nan")


def bootstrap(stat: Callable[[Sequence[Record]], float], rs: Sequence[Record], iters: int = 1000,
              seed: int = 0) -> Tuple[float, float, float]:
    rng = random.Random(seed)
    n = len(rs)
    vals = []
    for _ in range(iters):
        v = stat([rs[rng.randrange(n)] for _ in range(n)])
        if not math.isnan(v):
            vals.append(v)
    vals.sort()
    if not vals:
        return stat(rs), float("nan"), float("nan")
    return stat(rs), vals[int(0.025 * len(vals))], vals[max(0, int(0.975 * len(vals)) - 1)]


def p0_checks(rs: Sequence[Record], iters: int = 1000, rho_min: float = 0.3, r2_min: float = 0.7,
              mono_min: float = 0.6) -> Dict[str, dict]:
    a = bootstrap(lambda s: spearman([r.eta for r in s], [r.speedup for r in s]), rs, iters)
    b = bootstrap(residual_r2, rs, iters)
    c = bootstrap(monotone_fraction, rs, iters)

    def verdict(v, lo, thr):
        return "PASS" if lo >= thr else ("WEAK" if v >= thr else "FAIL")
    return {"a": {"spearman": a[0], "ci": a[1:], "n": len(rs), "verdict": verdict(a[0], a[1], rho_min)},
            "b": {"r2": b[0], "ci": b[1:], "verdict": verdict(b[0], b[1], r2_min)},
            "c": {"monotone_frac": c[0], "ci": c[1:], "verdict": verdict(c[0], c[1], mono_min)}}


def leave_one_family_out(rs: Sequence[Record]) -> Dict[str, float]:
    fams = sorted({r.family for r in rs})
    out = {}
    for f in fams:
        tr = [r for r in rs if r.family != f]
        te = [r for r in rs if r.family == f]
        if len(tr) < 5 or len(te) < 3:
            continue
        coef, _ = ols_r2(*_design(tr))
        X, y = _design(te)
        res = y - X @ coef
        tot = ((y - y.mean()) ** 2).sum()
        out[f] = float(1 - (res ** 2).sum() / tot) if tot > 0 else float("nan")
    return out


def attained_fraction(flops: float, bytes_: float, measured_ms: float, peaks: dict, dtype: str = "bf16") -> dict:
    from .rooflines import peak_flops
    t_c = flops / peak_flops(peaks, dtype) * 1e3
    t_m = bytes_ / peaks["hbm_bytes_per_s"] * 1e3
    return {"compute_frac": t_c / measured_ms, "memory_frac": t_m / measured_ms,
            "eta": max(t_c, t_m) / measured_ms, "bound": "compute" if t_c >= t_m else "memory"}


def bottleneck_from_counters(c: Dict[str, float]) -> str:
    """Limiter of one kernel from ncu counters (percent metrics in [0, 100])."""
    from ..verifier.pmc import counter
    tensor = counter(c, "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active") or 0.0
    dram = counter(c, "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed") or 0.0
    sm = counter(c, "sm__throughput.avg.pct_of_peak_sustained_elapsed") or 0.0
    dur_ns = counter(c, "gpu__time_duration.sum") or 0.0
    if dur_ns and dur_ns < 5000:
        return "launch"
    if tensor >= 60:
        return "tensor"
    if dram >= 60:
        return "dram"
    if sm >= 60:
        return "sm_issue"
    return "latency"
