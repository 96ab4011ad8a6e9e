"""Competitor anchor for the curriculum: per task, how far this policy is
behind a strong external solver (a teacher model's best verified speedups).

``competitor_regret(ours, theirs)`` = clip(1 - our_best / their_best, 0, 1);
a task where the competitor has no verified win gets no entry (the proposer
then uses its plain score). ``from_records`` builds the map from JSONL win
records (``task_id``, ``speedup``, ``source``) such as the teacher datasets.
``build_competitor_scores`` mines the teacher's own verified datagen records
(wins and ranked groups) into a per-task strength in [0, 1] (log speedup over
a high percentile) or, given our best speedups, the regret against it; every
failure (missing files, bad lines) only makes the map smaller.

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


# ----------------------------------------------------------------------------- mined from verified data
def _percentile(vals, q: float) -> float:
    v = sorted(vals)
    if not v:
        return float("nan")
    x = (len(v) - 1) * min(1.0, max(0.0, q))
    lo, hi = int(math.floor(x)), int(math.ceil(x))
    return v[lo] + (v[hi] - v[lo]) * (x - lo)


def mine_teacher_speedups(paths: Iterable[str], *, min_snr_db: Optional[float] = None) -> Dict[str, float]:
    """Best verified speedup per task found in datagen records written by the
    teacher: a win's ``speedup``; a ranked group's correct candidates'
    ``parent_wall_us / wall_us``. Unreadable files and malformed lines are
    skipped (the result is simply smaller)."""
    best: Dict[str, float] = {}

    def bump(tid, s):
        try:
            s = float(s)
        except (TypeError, ValueError):
            return
        if tid and math.isfinite(s) and s > best.get(tid, 0.0):
            best[tid] = s
    for p in paths:
        try:
            fh = open(p)
        except OSError:
            continue
        with fh:
            for line in fh:
                try:
                    r = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if not isinstance(r, dict):
                    continue
                if r.get("type") == "win":
                    bump(r.get("task_id"), r.get("speedup"))
                elif r.get("type") == "ranked_group":
                    base = r.get("parent_wall_us")
                    for c in r.get("candidates") or []:
                        if not c.get("correct") or not c.get("wall_us") or not base:
                            continue
                        if min_snr_db is not None and (c.get("snr_db") is None or c["snr_db"] < min_snr_db):
                            continue
                        bump(r.get("task_id"), base / c["wall_us"])
    return best


def strength_scores(best: Mapping[str, float], *, ref_percentile: float = 0.95,
                    min_ref_speedup: float = 2.0) -> Dict[str, float]:
    """Competitor strength per task in [0, 1]: log(max(s, 1)) / log(S_ref) with
    S_ref the ``ref_percentile`` of the best speedups (at least
    ``min_ref_speedup``). Log because speedups compound; the percentile keeps
    one outlier from flattening every other task; s <= 1 (no headroom) maps to 0."""
    vals = [v for v in best.values() if v > 0 and math.isfinite(v)]
    if not vals:
        return {}
    ref = max(min_ref_speedup, _percentile(vals, ref_percentile))
    return {t: max(0.0, min(1.0, math.log(max(s, 1.0)) / math.log(ref))) for t, s in best.items()}


def build_competitor_scores(teacher_paths: Iterable[str], ours: Optional[Mapping[str, float]] = None,
                            **kw) -> Dict[str, float]:
    """The proposer's competitor map from verified teacher data: the teacher's
    strength per task, or, when our own best speedups are known, the regret
    against the teacher (tasks where we already match it drop to 0)."""
    best = mine_teacher_speedups(teacher_paths)
    if ours:
        return competitor_regret(ours, best)
    return strength_scores(best, **kw)


def save_scores(scores: Mapping[str, float], path: str) -> None:
    with open(path, "w") as f:
        json.dump({k: round(float(v), 6) for k, v in sorted(scores.items())}, f, indent=1)


def load_scores(path: str) -> Dict[str, float]:
    """{} when the file is missing or malformed (the proposer then ignores the anchor)."""
    try:
        with open(path) as f:
            d = json.load(f)
    except (OSError, json.JSONDecodeError):
        return {}
    out = {}
    for k, v in (d.items() if isinstance(d, dict) else []):
        try:
            v = float(v)
        except (TypeError, ValueError):
            continue
        if math.isfinite(v):
            out[str(k)] = max(0.0, min(1.0, v))
    return out


def summarize(scores: Mapping[str, float]) -> Dict[str, float]:
    v = sorted(scores.values())
    if not v:
        return {"tasks": 0}
    return {"tasks": len(v), "mean": sum(v) / len(v), "median": _percentile(v, 0.5),
            "saturated": sum(1 for x in v if x >= 0.999), "zero": sum(1 for x in v if x <= 0.0)}
