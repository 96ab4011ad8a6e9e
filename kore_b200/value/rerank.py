"""The GRPO-facing ranking contract of the value model.

``score_candidates(sources, task=None, model=None)`` returns one score per
candidate (higher = bench first) and ``rank_candidates`` the best-first
indices. With a trained model the score is its utility
p_compile * p_snr * exp(E[log speedup]) (or its pairwise rank score); without
one, or when the model is degenerate on this set (a near-constant utility over
distinct sources, which would make the prior uninformative), a hand-written
schedule heuristic for sm_100a Triton kernels is used: tensor-core dot
products, 64-multiple tiles, moderate warp / stage counts, an fp32
accumulator, masked edges, a K loop, exp2. A bounded structural tie-breaker
keeps distinct sources from collapsing onto one score.

Replay validation: ``spearman`` between predicted and measured speedups and
``benches_to_best`` (how many benches a ranking needs before it reaches the
fastest correct candidate, against the expected number for a random order).

Reference behaviour: kore/value/rerank.py:1-262, train_value.py.
"""
from __future__ import annotations

import hashlib
import math
import re
from typing import List, Optional, Sequence

import numpy as np

from .model import ValueModel

_DEFAULT: Optional[ValueModel] = None


def load_default_model(path: Optional[str] = None) -> Optional[ValueModel]:
    global _DEFAULT
    if path:
        with open(path) as f:
            _DEFAULT = ValueModel.from_json(f.read())
    return _DEFAULT


def _int(src: str, name: str) -> Optional[int]:
    m = re.search(rf"\b{name}\s*[=:]\s*(\d+)", src)
    return int(m.group(1)) if m else None


def heuristic_score(src: str) -> float:
    s = src or ""
    sc = 0.0
    if "tl.dot(" in s:
        sc += 1.0
    for k in ("BM", "BN", "BK", "BLOCK_M", "BLOCK_N", "BLOCK_K", "BLOCK"):
        v = _int(s, k)
        if v is not None:
            sc += 0.25 if v % 64 == 0 else (-0.25 if v < 16 else 0.0)
    w = _int(s, "num_warps")
    if w is not None:
        sc += 0.25 if w in (4, 8) else -0.1
    st = _int(s, "num_stages")
    if st is not None:
        sc += 0.25 if 2 <= st <= 4 else -0.1
    if re.search(r"tl\.zeros\([^\n]*float32", s):
        sc += 0.25
    if "mask=" in s:
        sc += 0.2
    if re.search(r"for \w+ in (tl\.)?range\(", s):
        sc += 0.2
    if "exp2" in s:
        sc += 0.1
    if "tl.atomic" in s:
        sc -= 0.1
    return sc


def _tiebreak(src: str) -> float:
    return int(hashlib.sha1((src or "").encode()).hexdigest()[:6], 16) / float(1 << 24) * 1e-3


def _degenerate(vals: np.ndarray, sources: Sequence[str]) -> bool:
    distinct = len(set(sources)) > 1
    return distinct and float(np.ptp(vals)) < 1e-6 * max(1.0, float(np.abs(vals).max()))


def score_candidates(sources: Sequence[str], task=None, model: Optional[ValueModel] = None) -> List[float]:
    sources = list(sources)
    if not sources:
        return []
    model = model if model is not None else _DEFAULT
    from .features import task_meta
    meta = task_meta(task)
    if model is not None:
        try:
            p = model.predict(model.featurize(sources, meta))
            vals = np.asarray(p.get("rank_score", p["utility"]), dtype=np.float64)
            if np.all(np.isfinite(vals)) and not _degenerate(vals, sources):
                return [float(v) + _tiebreak(s) for v, s in zip(vals, sources)]
        except Exception:  # noqa: BLE001 - a broken model falls back to the heuristic
            pass
    return [heuristic_score(s) + _tiebreak(s) for s in sources]


def rank_candidates(sources: Sequence[str], task=None, model: Optional[ValueModel] = None) -> List[int]:
    sc = score_candidates(sources, task, model)
    return sorted(range(len(sc)), key=lambda i: -sc[i])


# ----------------------------------------------------------------------------- replay validation
def spearman(a: Sequence[float], b: Sequence[float]) -> float:
    n = len(a)
    if n < 2:
        return float("nan")

    def ranks(x):
        order = sorted(range(n), key=lambda i: x[i])
        r = [0.0] * n
        i = 0
        while i < n:
            j = i
            while j + 1 < n and x[order[j + 1]] == x[order[i]]:
                j += 1
            for k in range(i, j + 1):
                r[order[k]] = (i + j) / 2.0
            i = j + 1
        return r
    ra, rb = ranks(list(a)), ranks(list(b))
    ma, mb = sum(ra) / n, sum(rb) / n
    cov = sum((x - ma) * (y - mb) for x, y in zip(ra, rb))
    va = math.sqrt(sum((x - ma) ** 2 for x in ra))
    vb = math.sqrt(sum((y - mb) ** 2 for y in rb))
    return cov / (va * vb) if va and vb else float("nan")


def benches_to_best(order: Sequence[int], speedups: Sequence[Optional[float]]) -> Optional[int]:
    """1-based position in ``order`` of the fastest correct candidate (None
    when no candidate is correct)."""
    good = [(s, i) for i, s in enumerate(speedups) if s is not None]
    if not good:
        return None
    best = max(good)[1]
    return list(order).index(best) + 1


def expected_random_benches(n: int) -> float:
    return (n + 1) / 2.0


def top_k_recall(scores: Sequence[float], speedups: Sequence[Optional[float]], k: int) -> float:
    """1.0 when the fastest correct candidate is among the ``k`` highest scores
    (0.0 otherwise; nan when nothing is correct)."""
    order = sorted(range(len(scores)), key=lambda i: -scores[i])
    pos = benches_to_best(order, speedups)
    return float("nan") if pos is None else float(pos <= k)


def groupwise_spearman(score_fn, groups: Sequence[Sequence[dict]]) -> float:
    """Mean within-group Spearman correlation between ``score_fn(rows)`` and
    the measured speedups of the correct rows (groups with < 2 correct rows
    are skipped)."""
    vals = []
    for g in groups:
        rows = [r for r in g if r.get("speedup") is not None]
        if len(rows) < 2:
            continue
        rho = spearman(score_fn(rows), [r["speedup"] for r in rows])
        if rho == rho:
            vals.append(rho)
    return sum(vals) / len(vals) if vals else float("nan")
