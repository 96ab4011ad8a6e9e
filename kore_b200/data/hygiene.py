"""Dataset hygiene: near-duplicate removal (MinHash over code shingles),
decontamination against held-out tasks / eval prompts, and a quality filter
(parsable kernel, bounded length, no hack patterns). Reference parity:
kore/data/dedup.py, decontam.py, corpus_quality.py, curate.py."""
from __future__ import annotations

import hashlib
import re
from typing import Callable, Iterable, List, Sequence, Set

from ..reward.reward import scan_for_hacks

_TOK = re.compile(r"[A-Za-z_]\w*|\d+|[^\s\w]")


def shingles(text: str, n: int = 5) -> Set[str]:
    toks = _TOK.findall(text or "")
    return {" ".join(toks[i:i + n]) for i in range(max(1, len(toks) - n + 1))}


def minhash(text: str, k: int = 64, n: int = 5) -> List[int]:
    sh = shingles(text, n) or {""}
    sig = []
    for i in range(k):
        salt = str(i).encode()
        sig.append(min(int.from_bytes(hashlib.blake2b(salt + s.encode(), digest_size=8).digest(), "little")
                       for s in sh))
    return sig


def jaccard_est(a: Sequence[int], b: Sequence[int]) -> float:
    return sum(x == y for x, y in zip(a, b)) / max(1, len(a))


def dedup(items: Iterable, key: Callable = lambda x: x, threshold: float = 0.9, k: int = 64) -> List:
    """Keep the first of every group of near-duplicates (estimated Jaccard >= threshold)."""
    kept, sigs = [], []
    bands = {}
    for it in items:
        sig = minhash(key(it), k)
        cand = set()
        for b in range(0, k, 8):
            cand |= bands.get((b, tuple(sig[b:b + 8])), set())
        if any(jaccard_est(sig, sigs[j]) >= threshold for j in cand):
            continue
        idx = len(kept)
        kept.append(it)
        sigs.append(sig)
        for b in range(0, k, 8):
            bands.setdefault((b, tuple(sig[b:b + 8])), set()).add(idx)
    return kept


def decontaminate(items: Iterable, heldout_texts: Sequence[str], key: Callable = lambda x: x,
                  threshold: float = 0.5) -> List:
    held = [minhash(t) for t in heldout_texts]
    return [it for it in items if all(jaccard_est(minhash(key(it)), h) < threshold for h in held)]


def quality_ok(kernel: str, max_chars: int = 40000) -> bool:
    if not kernel or len(kernel) > max_chars:
        return False
    if scan_for_hacks(kernel):
        return False
    try:
        compile(kernel, "<kernel>", "exec")
    except SyntaxError:
        return False
    return True
