"""Frontier scoring of curriculum tasks.

    score = w_learn * learnability + w_regret * regret + w_novel * novelty
            (+ w_comp * competitor_regret * learnability)

* learnability = 4 p (1 - p) from the archive's solve-rate estimate; with
  evidence, a task whose rate is below ``p_min`` (hopeless for now) or above
  ``p_max`` (mastered) scores 0 on every term: it is outside the zone of
  proximal development.
* regret: the unrealised speedup headroom of the task (archive).
* novelty: mean niche (Hamming) distance to the occupied niches, normalised
  to [0, 1]; an unexplored region of the behaviour space is novel.
* competitor anchor (optional): a map ``{task_id: regret vs. a strong external
  solver in [0, 1]}``; missing, non-finite or out-of-range entries are ignored
  (the plain score is used), so without a map the score is unchanged.

Ties break on task id, so the ranking is identical on every rank.
Reference behaviour: kore/openended/proposer.py:118-307.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Sequence, Tuple

from .archive import DescriptorStats, TaskArchive
from .task_space import niche_distance


@dataclass
class FrontierWeights:
    learn: float = 1.0
    regret: float = 0.5
    novel: float = 0.3
    competitor: float = 0.0
    p_min: float = 0.05
    p_max: float = 0.95


class Proposer:
    def __init__(self, w_learn: float = 1.0, w_regret: float = 0.5, w_novel: float = 0.3,
                 competitor: Optional[Mapping[str, float]] = None, w_competitor: float = 0.5,
                 p_min: float = 0.05, p_max: float = 0.95):
        self.w = FrontierWeights(w_learn, w_regret, w_novel, w_competitor if competitor else 0.0, p_min, p_max)
        self.competitor = dict(competitor or {})

    def novelty(self, e: DescriptorStats, occupied: Sequence[Tuple]) -> float:
        if not occupied:
            return 1.0
        n = e.desc.niche()
        return sum(niche_distance(n, c) for c in occupied) / (len(occupied) * len(n))

    def _competitor(self, tid: str) -> float:
        v = self.competitor.get(tid)
        try:
            v = float(v)
        except (TypeError, ValueError):
            return 0.0
        return v if math.isfinite(v) and 0.0 <= v <= 1.0 else 0.0

    def score(self, e: DescriptorStats, occupied=None) -> float:
        if isinstance(occupied, dict):            # earlier signature: {niche: times seen}
            occupied = [c for c, k in occupied.items() if k > 0]
        occupied = occupied or []
        w = self.w
        if e.has_evidence and not (w.p_min < e.p < w.p_max):
            return 0.0
        learn = e.informativeness
        s = w.learn * learn + w.regret * e.regret + w.novel * self.novelty(e, occupied)
        if w.competitor:
            s += w.competitor * self._competitor(e.desc.task_id) * learn
        return s

    def rank(self, archive: TaskArchive, candidates: Optional[Sequence[str]] = None,
             extra_occupied: Sequence[Tuple] = ()) -> List[Tuple[float, str]]:
        occ = list(archive.occupied()) + list(extra_occupied)
        ids = candidates if candidates is not None else list(archive.entries)
        scored = [(self.score(archive.entries[t], occ), t) for t in ids if t in archive.entries]
        return sorted(scored, key=lambda x: (-x[0], x[1]))


def proposal_table(archive: TaskArchive, proposer: Proposer, k: int = 10) -> List[Dict[str, object]]:
    """The top ``k`` of the frontier with the terms of their scores (for logs)."""
    occ = archive.occupied()
    out = []
    for s, tid in proposer.rank(archive)[:k]:
        e = archive.entries[tid]
        out.append({"task_id": tid, "score": round(s, 4), "p": round(e.p, 3), "regret": round(e.regret, 3),
                    "novelty": round(proposer.novelty(e, occ), 3), "attempts": e.attempts})
    return out
