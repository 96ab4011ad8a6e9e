"""CoevolutionController: the GRPO-facing curriculum.

``next_task_id(k)`` serves task ids from a queue refilled by the proposer's
frontier ranking over the allowed (held-out-free) tasks. A fraction
``explore`` of each refill comes from mutation: a frontier descriptor moved
to a neighbouring point of the task space, mapped back to the nearest
registered task not already queued. With ``mint`` on, every
``mint_every``-th refill asks the task minter for new correct-by-construction
tasks and adds them to the space (a mint that fails its gate is skipped).

Distributed determinism: all randomness comes from ``seed`` and the refill
counter, and ``record_batch`` all-gathers the per-rank outcomes before
updating the archive, so every rank holds the same archive and serves the
same ids.

Reference behaviour: kore/openended/controller.py:41-326.
"""
from __future__ import annotations

import random
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from .archive import TaskArchive
from .proposer import Proposer
from .task_space import TaskDescriptor, TaskSpace, descriptor_of


class CoevolutionController:
    def __init__(self, space: Optional[TaskSpace] = None, seed: int = 0, proposer: Optional[Proposer] = None, *,
                 allowed: Optional[Iterable[str]] = None, batch: int = 8, explore: float = 0.25,
                 mint: bool = False, mint_every: int = 4, mint_batch: int = 6, ctx=None):
        self.space = space or TaskSpace(allowed=allowed)
        self.allowed = set(allowed) if allowed is not None else None
        self.archive = TaskArchive()
        for d in self.space.items:
            self.archive.add(d)
        self.proposer = proposer or Proposer()
        self.seed, self.batch, self.explore = seed, max(1, batch), explore
        self.mint, self.mint_every, self.mint_batch = mint, max(1, mint_every), mint_batch
        self.ctx = ctx
        self.refills = 0
        self.queue: List[str] = []
        self.served: Dict[str, int] = {}
        self.minted: List[str] = []

    # ------------------------------------------------------------------ serving
    def _rng(self) -> random.Random:
        return random.Random(self.seed * 1_000_003 + self.refills)

    def _refill(self) -> None:
        rng = self._rng()
        self.refills += 1
        if self.mint and self.refills % self.mint_every == 0:
            self._mint(rng)
        ranked = [t for _, t in self.proposer.rank(self.archive)]
        if not ranked:
            return
        n_exp = int(round(self.explore * self.batch))
        picks = ranked[: max(1, self.batch - n_exp)]
        for _ in range(n_exp * 3):
            if len(picks) >= self.batch:
                break
            base = self.space.by_id(rng.choice(ranked[: max(1, self.batch)]))
            if base is None:
                continue
            near = self.space.nearest(self.space.mutate(base, rng), exclude=picks)
            if near is not None and near.task_id not in picks:
                picks.append(near.task_id)
        for t in ranked:
            if len(picks) >= self.batch:
                break
            if t not in picks:
                picks.append(t)
        self.queue.extend(picks)

    def next_task_id(self, k: int = 1) -> List[str]:
        out: List[str] = []
        guard = 0
        while len(out) < k and guard < 4 * k + 8:
            guard += 1
            if not self.queue:
                self._refill()
                if not self.queue:
                    break
            out.append(self.queue.pop(0))
        for t in out:
            self.served[t] = self.served.get(t, 0) + 1
        return out

    def resolve_task(self, tid: str):
        from ..tasks.registry import get_task
        return get_task(tid)

    # ------------------------------------------------------------------ feedback
    def record(self, tid: str, success, regret: Optional[float] = None, speedup: Optional[float] = None,
               ceiling: Optional[float] = None) -> None:
        if tid not in self.archive.entries:
            d = self.space.by_id(tid)
            if d is None:
                return
            self.archive.add(d)
        self.archive.record(tid, success, regret=regret, speedup=speedup, ceiling=ceiling,
                            score=lambda e: self.proposer.score(e, self.archive.occupied()))

    def record_batch(self, results: Sequence[Tuple[str, float, Optional[float]]]) -> None:
        """(task_id, solve_rate, best_speedup) from this rank; gathered over
        ranks and merged per task (mean solve rate, max speedup) in id order."""
        allr = [list(results)]
        if self.ctx is not None and getattr(self.ctx, "world", 1) > 1:
            allr = self.ctx.all_gather_object(list(results))
        merged: Dict[str, List] = {}
        for rank_res in allr:
            for tid, rate, sp in rank_res:
                m = merged.setdefault(tid, [0.0, 0, None])
                m[0] += float(rate)
                m[1] += 1
                if sp is not None and (m[2] is None or sp > m[2]):
                    m[2] = float(sp)
        for tid in sorted(merged):
            s, n, sp = merged[tid]
            self.record(tid, s / n, speedup=sp)

    # ------------------------------------------------------------------ minting
    def _mint(self, rng: random.Random) -> None:
        from ..tasks.registry import get_task
        from .minter import TaskMinter
        try:
            new = TaskMinter(seed=rng.randrange(1 << 30)).mint(self.mint_batch)
        except Exception:                            # a failed mint never stops training
            return
        for tid in new:
            try:
                d = descriptor_of(get_task(tid))
            except Exception:
                d = None
            if d is not None:
                self.space.add(d)
                self.archive.add(d)
                self.minted.append(tid)

    # ------------------------------------------------------------------ checkpoint
    def state_dict(self) -> Dict[str, object]:
        return {"refills": self.refills, "queue": list(self.queue), "served": dict(self.served),
                "stats": {t: [e.attempts, e.succ_w, e.tot_w, e.best_speedup, e.regret]
                          for t, e in self.archive.entries.items() if e.attempts}}

    def load_state_dict(self, st: Dict[str, object]) -> None:
        self.refills = int(st.get("refills", 0))
        self.queue = list(st.get("queue", []))
        self.served = dict(st.get("served", {}))
        for t, (a, sw, tw, bs, rg) in dict(st.get("stats", {})).items():
            if t in self.archive.entries:
                e = self.archive.entries[t]
                e.attempts, e.succ_w, e.tot_w, e.best_speedup, e.regret = a, sw, tw, bs, rg
                self.archive._place(e, lambda x: x.informativeness + 0.5 * x.regret)


# earlier name, same object
CurriculumController = CoevolutionController
