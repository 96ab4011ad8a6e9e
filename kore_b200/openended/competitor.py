"""Competitor anchor for the curriculum: per task, how far this policy is
behind a strong external solver (a teacher model's best verified speedups).

``competitor_regret(ours, theirs)`` = clip(1 - our_best / their_best, 0, 1);
a task where the competitor has no verified win gets no entry (the proposer
then uses its plain score). ``from_records`` builds the map from JSONL win
records (``task_id``, ``speedup``, ``source``) such as the teacher datasets.

Reference behaviour: kore/openended/opus_baseline.py:1-369.
"""
from __future__ import annotations

import json
import math
from typing import Dict, Iterable, Mapping, Optional


def competitor_regret(ours: Mapping[str, float], theirs: Mapping[str, float]) -> Dict[str, float]:
    out = {}
    for tid, t in theirs.items():
        try:
            t = float(t)
        except (TypeError, ValueError):
            continue
        if not math.isfinite(t) or t <= 0:
            continue
        o = float(ours.get(tid, 0.0) or 0.0)
        out[tid] = max(0.0, min(1.0, 1.0 - o / t))
    return out


def best_by_task(records: Iterable[dict], source: Optional[str] = None) -> Dict[str, float]:
    best: Dict[str, float] = {}
    for r in records:
        if source is not None and r.get("source") != source:
            continue
        if not r.get("correct", True):
            continue
        try:
            s = float(r.get("speedup"))
        except (TypeError, ValueError):
            continue
        tid = r.get("task_id")
        if tid and math.isfinite(s) and s > best.get(tid, 0.0):
            best[tid] = s
    return best


def from_records(path: str, *, ours: str = "policy", theirs: str = "teacher") -> Dict[str, float]:
    with open(path) as f:
        recs = [json.loads(l) for l in f if l.strip()]
    return competitor_regret(best_by_task(recs, ours), best_by_task(recs, theirs))
