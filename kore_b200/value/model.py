"""Value model over candidate kernels (numpy, no external deps).

Features: schedule knobs parsed from the source (tile sizes, warps, stages,
tl.dot use, exp vs exp2, vectorisation hints, masking, loop count, source
length) plus the task's roofline arithmetic intensity. Three heads:
p_compile and p_snr (logistic regressions) and E[log speedup] (ridge
regression); a RankNet pairwise head over feature differences. The ranking
score is p_compile * p_snr * exp(E[log su]). Trained from ranked-group
records; saved as JSON (never pickle). Reference parity:
kore/value/features.py:209-400, model.py:102-375, rerank.py:262,
replay_train.py:152.
"""
from __future__ import annotations

import argparse
import json
import math
import re
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

_KNOBS = ("BM", "BN", "BK", "BLOCK", "num_warps", "num_stages", "GROUP_SIZE_M")


def features(src: str, arith_intensity: float = 0.0) -> np.ndarray:
    f = []
    for k in _KNOBS:
        m = re.search(rf"\b{k}\s*[=:]\s*(\d+)", src or "")
        f.append(math.log2(int(m.group(1))) if m else 0.0)
    s = src or ""
    f += [float("tl.dot" in s), float("exp2" in s), float("multiple_of" in s or "max_contiguous" in s),
          float("mask=" in s), float(s.count("for ")), math.log1p(len(s)), math.log1p(max(0.0, arith_intensity)),
          1.0]
    return np.asarray(f, dtype=np.float64)


def _sig(z):
    return 1.0 / (1.0 + np.exp(-np.clip(z, -30, 30)))


def _logreg(X, y, l2=1e-2, iters=300, lr=0.5):
    w = np.zeros(X.shape[1])
    for _ in range(iters):
        g = X.T @ (_sig(X @ w) - y) / len(y) + l2 * w
        w -= lr * g
    return w


class ValueModel:
    """``featurizer``: "v2" (schedule of Triton or CUDA sources plus the task
    context, :mod:`kore_b200.value.features`) for new models; "v1" (the
    Triton-knob vector of :func:`features`) for models saved before it."""

    def __init__(self, featurizer: str = "v2"):
        self.w_compile = self.w_snr = self.w_speed = self.w_rank = None
        self.mu = self.sd = None
        self.featurizer = featurizer

    def featurize(self, sources: Sequence[str], meta: Optional[dict] = None) -> np.ndarray:
        if self.featurizer == "v1":
            ai = float((meta or {}).get("intensity") or 0.0)
            return np.stack([features(s, ai) for s in sources])
        from .features import featurize_many
        return featurize_many(sources, meta)

    def fit_groups(self, groups: Sequence[Sequence[dict]]) -> "ValueModel":
        """Fit from ranked groups of rows {"source", "compiled", "correct",
        "speedup" (None unless correct), "meta"}: the three heads on every row
        and the pairwise head on every (faster correct, slower or incorrect)
        pair inside a group."""
        F, comp, corr, ls, pairs = [], [], [], [], []
        for g in groups:
            i0 = len(F)
            for r in g:
                F.append(self.featurize([r.get("source", "")], r.get("meta"))[0])
                comp.append(bool(r.get("compiled")))
                corr.append(bool(r.get("correct")))
                su = r.get("speedup")
                ls.append(math.log(su) if su else 0.0)
            for a in range(len(g)):
                for b in range(len(g)):
                    sa, sb = g[a].get("speedup"), g[b].get("speedup")
                    if sa is not None and (sb is None or sa > sb * 1.02):
                        pairs.append((i0 + a, i0 + b))
        if not F:
            raise ValueError("no training rows")
        return self.fit(np.stack(F), np.array(comp), np.array(corr), np.array(ls), pairs)

    def _x(self, F: np.ndarray) -> np.ndarray:
        return (F - self.mu) / self.sd if self.mu is not None else F

    def fit(self, F: np.ndarray, compiled: np.ndarray, correct: np.ndarray, log_speed: np.ndarray,
            pairs: Sequence[Tuple[int, int]] = ()) -> "ValueModel":
        self.mu = F.mean(0)
        self.sd = F.std(0) + 1e-6
        self.mu[-1], self.sd[-1] = 0.0, 1.0
        X = self._x(F)
        self.w_compile = _logreg(X, compiled.astype(float))
        self.w_snr = _logreg(X, correct.astype(float))
        m = correct.astype(bool)
        if m.sum() >= 2:
            # throughput weighting: fast kernels dominate the fit (weight = max(speedup, 0.1))
            Xm = X[m]
            wts = np.maximum(np.exp(log_speed[m]), 0.1)
            A = Xm.T @ (Xm * wts[:, None]) + 1e-1 * np.eye(X.shape[1])
            self.w_speed = np.linalg.solve(A, Xm.T @ (wts * log_speed[m]))
        else:
            self.w_speed = np.zeros(X.shape[1])
        if pairs:
            D = np.stack([X[i] - X[j] for i, j in pairs])
            self.w_rank = _logreg(D, np.ones(len(pairs)))
        return self

    def predict(self, F: np.ndarray) -> Dict[str, np.ndarray]:
        X = self._x(F)
        pc, ps = _sig(X @ self.w_compile), _sig(X @ self.w_snr)
        ls = X @ self.w_speed
        out = {"p_compile": pc, "p_snr": ps, "log_speedup": ls, "utility": pc * ps * np.exp(ls)}
        if self.w_rank is not None:
            out["rank_score"] = X @ self.w_rank
        return out

    def to_json(self) -> str:
        d = {k: (v.tolist() if v is not None else None) for k, v in
             dict(w_compile=self.w_compile, w_snr=self.w_snr, w_speed=self.w_speed,
                  w_rank=self.w_rank, mu=self.mu, sd=self.sd).items()}
        d["featurizer"] = self.featurizer
        return json.dumps(d)

    @classmethod
    def from_json(cls, s: str) -> "ValueModel":
        d = json.loads(s)
        m = cls(featurizer=d.pop("featurizer", "v1"))
        for k, v in d.items():
            setattr(m, k, None if v is None else np.asarray(v))
        return m


def refit_online(buffer: List[List[dict]], new_groups: Sequence[Sequence[dict]], max_groups: int = 2000,
                 featurizer: str = "v2") -> ValueModel:
    """Append ``new_groups`` (measured this step) to the replay ``buffer``
    (oldest dropped beyond ``max_groups``) and refit a model on it."""
    buffer.extend(list(g) for g in new_groups)
    del buffer[: max(0, len(buffer) - max_groups)]
    return ValueModel(featurizer).fit_groups(buffer)


def rank_candidates(model: ValueModel, sources: Sequence[str], ai: float = 0.0) -> List[int]:
    F = model.featurize(sources, {"intensity": ai})
    p = model.predict(F)
    key = p.get("rank_score", p["utility"])
    return list(np.argsort(-key))


def train_from_groups(paths: Sequence[str], featurizer: str = "v2") -> ValueModel:
    """Fit from RankedGroupRecord JSONL files: the heads on every candidate
    (speedup = the parent's wall time over the candidate's) and the pairwise
    head on the records' own preference pairs."""
    from ..data.schemas import RankedGroupRecord, read_records
    from .features import meta_from_record
    m = ValueModel(featurizer)
    F, comp, corr, ls, pairs = [], [], [], [], []
    metas: Dict[str, dict] = {}
    for p in paths:
        for r in read_records(p, RankedGroupRecord):
            if r.task_id not in metas:
                metas[r.task_id] = meta_from_record(r.task_id, r.operation, r.shape)
            base = r.parent_wall_us
            idx0 = len(F)
            for c in r.candidates:
                F.append(m.featurize([c.get("source", "")], metas[r.task_id])[0])
                comp.append(c.get("snr_db") is not None)
                corr.append(bool(c.get("correct")))
                w = c.get("wall_us")
                ls.append(math.log(base / w) if (base and w) else 0.0)
            pairs += [(idx0 + a, idx0 + b) for a, b in r.preferences]
    if not F:
        raise ValueError("no training rows")
    return m.fit(np.stack(F), np.array(comp), np.array(corr), np.array(ls), pairs)
