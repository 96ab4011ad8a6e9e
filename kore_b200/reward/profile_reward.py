"""Counter-relative dense efficiency score (ncu counters, candidate vs baseline).

Score in [0, 1]: 0.5 + 0.5 * tanh of the log-ratio of the baseline's to the
candidate's stall fraction and DRAM traffic, averaged, so doing the same work
with fewer stalls / fewer bytes than the vendor kernel scores above 0.5.
Behavioural parity (different counters): kore/reward/profile_reward.py:98-200.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

from .whitebox import stall_frac_from_counters


def _bytes(c: dict) -> Optional[float]:
    r, w = c.get("dram__bytes_read.sum"), c.get("dram__bytes_write.sum")
    if r is None and w is None:
        return None
    return float(r or 0) + float(w or 0)


@dataclass
class ProfileMetrics:
    stall_cand: Optional[float]
    stall_ref: Optional[float]
    bytes_cand: Optional[float]
    bytes_ref: Optional[float]
    score: Optional[float]


def _ratio_term(ref, cand):
    if ref is None or cand is None or ref <= 0 or cand <= 0:
        return None
    return 0.5 + 0.5 * math.tanh(math.log(ref / cand))


def profile_efficiency_score(cand: dict, ref: dict) -> Optional[float]:
    terms = [t for t in (_ratio_term(stall_frac_from_counters(ref), stall_frac_from_counters(cand)),
                         _ratio_term(_bytes(ref), _bytes(cand))) if t is not None]
    return sum(terms) / len(terms) if terms else None


def roofline_dense_score(t_min_ms: Optional[float], measured_ms: Optional[float]) -> Optional[float]:
    """Attainment T_min / T_meas clamped to [0, 1]."""
    if not t_min_ms or not measured_ms or measured_ms <= 0:
        return None
    return max(0.0, min(1.0, t_min_ms / measured_ms))


def profile_metrics(cand: dict, ref: dict) -> ProfileMetrics:
    return ProfileMetrics(stall_frac_from_counters(cand), stall_frac_from_counters(ref), _bytes(cand),
                          _bytes(ref), profile_efficiency_score(cand, ref))
