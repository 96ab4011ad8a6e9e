"""Dataset assembly aligned with the RL objective.

* ``leakage_split``: train / val / test by whole groups (default key:
  (family, arch)), assigned by a stable hash, so near-identical records of one
  operator family never straddle the split; the registry's held-out tasks are
  removed first (the final authority).
* ``filter_trivial_wins``: optimisation wins must be genuinely faster than
  their parent (the same speedup objective the GRPO reward optimises).
* ``build_multicap``: the multi-capability SFT mix (repair, wins, QA,
  agentic, general replay) with a cap and a weight per capability,
  deterministic for a seed.
* ``dpo_with_hard_negatives``: DPO pairs with a floor on the fraction whose
  rejected side is a reward-hacking kernel (so the policy learns to prefer an
  honest kernel over a fast-looking hack), topping up from the negatives pool.
* ``coverage``: records per family and per task, and the training tasks with
  no record at all.

Reference behaviour: kore/data/assemble.py, build_datasets.py:124-686,
hard_negatives.py, coverage.py, mixing.py.
"""
from __future__ import annotations

import hashlib
import random
from collections import Counter
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple


def _bucket(key: str, seed: int) -> float:
    h = hashlib.sha1(f"{seed}:{key}".encode()).hexdigest()
    return int(h[:12], 16) / float(1 << 48)


def leakage_split(rows: Sequence[Dict], *, fractions: Tuple[float, float, float] = (0.9, 0.05, 0.05),
                  key: Optional[Callable[[Dict], str]] = None, heldout: Iterable[str] = (), seed: int = 0
                  ) -> Dict[str, List[Dict]]:
    if abs(sum(fractions) - 1.0) > 1e-9:
        raise ValueError("fractions must sum to 1")
    ho = set(heldout)
    key = key or (lambda r: f"{r.get('family', '')}|{r.get('arch', 'sm_100a')}")
    out = {"train": [], "val": [], "test": []}
    a, b = fractions[0], fractions[0] + fractions[1]
    for r in rows:
        if r.get("task_id") in ho:
            continue
        u = _bucket(key(r), seed)
        out["train" if u < a else ("val" if u < b else "test")].append(r)
    return out


def filter_trivial_wins(wins: Iterable, min_speedup: float = 1.02) -> List:
    return [w for w in wins if (getattr(w, "speedup", None) or 0.0) >= min_speedup]


def build_multicap(sources: Dict[str, Sequence[Dict]], caps: Dict[str, int],
                   weights: Optional[Dict[str, float]] = None, seed: int = 0) -> List[Dict]:
    """Per capability: shuffle, keep at most ``caps[kind]`` rows, tag
    ``_source`` and ``_weight``; the union is shuffled."""
    rng = random.Random(seed)
    out: List[Dict] = []
    for kind in sorted(sources):
        rows = list(sources[kind])
        rng.shuffle(rows)
        cap = caps.get(kind, len(rows))
        w = (weights or {}).get(kind, 1.0)
        for r in rows[:cap]:
            out.append({**r, "_source": kind, "_weight": w})
    rng.shuffle(out)
    return out


def dpo_with_hard_negatives(pairs: Sequence[Dict], negatives: Sequence[Dict], *, min_frac: float = 0.08,
                            seed: int = 0) -> List[Dict]:
    """``pairs``: {prompt, chosen, rejected, [hack]}; ``negatives``: pairs whose
    rejected side is a reward hack. Adds negatives until at least ``min_frac``
    of the result is hack-rejecting (when the pool allows)."""
    rng = random.Random(seed)
    out = list(pairs)
    have = sum(1 for p in out if p.get("hack"))
    pool = [dict(n, hack=True) for n in negatives]
    rng.shuffle(pool)
    while pool and have < min_frac * len(out):
        out.append(pool.pop())
        have += 1
    rng.shuffle(out)
    return out


def coverage(rows: Iterable[Dict], tasks: Sequence) -> Dict[str, object]:
    per_task = Counter(r.get("task_id") for r in rows)
    fam = {t.task_id: t.family for t in tasks}
    per_family: Counter = Counter()
    for tid, n in per_task.items():
        per_family[fam.get(tid, "unknown")] += n
    missing = sorted(t.task_id for t in tasks if per_task.get(t.task_id, 0) == 0)
    return {"records": sum(per_task.values()), "tasks_covered": sum(1 for t in tasks if per_task.get(t.task_id)),
            "tasks": len(tasks), "per_family": dict(per_family), "missing": missing}
