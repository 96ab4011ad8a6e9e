"""Open-ended curriculum over kernel tasks.

* ``TaskDescriptor`` / ``TaskSpace``: the space of candidate tasks (library
  ops x shapes x dtypes) with MAP-Elites features (family, arithmetic
  intensity bucket, size bucket).
* ``TaskArchive``: MAP-Elites of tasks scored by informativeness
  4p(1-p) (p = policy success rate, maximal at 0.5) plus regret against a
  reference solver.
* ``Proposer``: scores proposals by learnability + regret + novelty.
* ``CurriculumController``: deterministic frontier selection (identical on
  every rank given the same seed and history), ``record`` of outcomes.
* ``coevolve``: propose -> attempt -> update -> distill loop.
Reference parity: kore/openended/task_space.py:111-357, archive.py:28-149,
proposer.py:118-307, controller.py:41-326, coevolve.py:82-174.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

from ..analysis.rooflines import flops_bytes
from ..tasks.registry import all_tasks


@dataclass(frozen=True)
class TaskDescriptor:
    task_id: str
    family: str
    operation: str
    dtype: str
    dims: Tuple[Tuple[str, int], ...]

    def features(self) -> Tuple[str, int, int]:
        d = dict(self.dims)
        fb = flops_bytes(self.operation, d, self.dtype)
        ai = fb[0] / fb[1] if fb and fb[1] else 0.0
        size = 1
        for v in d.values():
            size *= max(1, v)
        return (self.family, int(math.log2(1 + ai)), int(math.log2(size)) // 4)


class TaskSpace:
    def __init__(self, tasks=None):
        self.items: List[TaskDescriptor] = []
        for t in (tasks or all_tasks()):
            sh = t.shape("primary") or (t.shapes[0] if t.shapes else None)
            if sh is None:
                continue
            self.items.append(TaskDescriptor(t.task_id, t.family, t.operation, t.dtype,
                                             tuple(sorted(sh.dims.items()))))

    def by_id(self, tid: str) -> Optional[TaskDescriptor]:
        return next((d for d in self.items if d.task_id == tid), None)


@dataclass
class ArchiveEntry:
    desc: TaskDescriptor
    attempts: int = 0
    successes: int = 0
    regret: float = 0.0

    @property
    def p(self) -> float:
        return (self.successes + 1) / (self.attempts + 2)       # Laplace-smoothed success rate

    @property
    def informativeness(self) -> float:
        return 4 * self.p * (1 - self.p)

    def score(self, w_regret: float = 0.5) -> float:
        return self.informativeness + w_regret * self.regret


class TaskArchive:
    def __init__(self):
        self.cells: Dict[tuple, ArchiveEntry] = {}
        self.entries: Dict[str, ArchiveEntry] = {}

    def add(self, d: TaskDescriptor) -> ArchiveEntry:
        e = self.entries.setdefault(d.task_id, ArchiveEntry(d))
        cell = d.features()
        cur = self.cells.get(cell)
        if cur is None or e.score() > cur.score():
            self.cells[cell] = e
        return e

    def record(self, tid: str, success: bool, regret: Optional[float] = None) -> None:
        e = self.entries[tid]
        e.attempts += 1
        e.successes += int(success)
        if regret is not None:
            e.regret = 0.8 * e.regret + 0.2 * regret
        cell = e.desc.features()
        if self.cells.get(cell) is None or e.score() >= self.cells[cell].score():
            self.cells[cell] = e

    def elites(self) -> List[ArchiveEntry]:
        return sorted(self.cells.values(), key=lambda e: -e.score())


class Proposer:
    def __init__(self, w_learn: float = 1.0, w_regret: float = 0.5, w_novel: float = 0.3):
        self.w = (w_learn, w_regret, w_novel)

    def score(self, e: ArchiveEntry, seen_cells: Dict[tuple, int]) -> float:
        novelty = 1.0 / math.sqrt(1 + seen_cells.get(e.desc.features(), 0))
        return self.w[0] * e.informativeness + self.w[1] * e.regret + self.w[2] * novelty


class CurriculumController:
    """Deterministic frontier: rank-identical choices for a given seed/history."""

    def __init__(self, space: Optional[TaskSpace] = None, seed: int = 0, proposer: Optional[Proposer] = None):
        self.space = space or TaskSpace()
        self.archive = TaskArchive()
        for d in self.space.items:
            self.archive.add(d)
        self.proposer = proposer or Proposer()
        self.rng = random.Random(seed)
        self.seen: Dict[tuple, int] = {}

    def next_task_id(self, k: int = 1) -> List[str]:
        ents = sorted(self.archive.entries.values(),
                      key=lambda e: (-self.proposer.score(e, self.seen), e.desc.task_id))
        out = [e.desc.task_id for e in ents[:k]]
        for t in out:
            c = self.archive.entries[t].desc.features()
            self.seen[c] = self.seen.get(c, 0) + 1
        return out

    def resolve_task(self, tid: str):
        from ..tasks.registry import get_task
        return get_task(tid)

    def record(self, tid: str, success: bool, regret: Optional[float] = None) -> None:
        self.archive.record(tid, success, regret)


def coevolve(controller: CurriculumController, attempt: Callable[[str], Tuple[bool, float]], rounds: int = 4,
             batch: int = 4, distill: Optional[Callable[[str, float], None]] = None) -> List[Tuple[str, bool]]:
    """propose -> attempt (returns success, best speedup) -> update -> distill."""
    log = []
    for _ in range(rounds):
        for tid in controller.next_task_id(batch):
            ok, speed = attempt(tid)
            controller.record(tid, ok, regret=max(0.0, 1.0 - speed) if ok else 1.0)
            if ok and distill is not None and speed > 1.0:
                distill(tid, speed)
            log.append((tid, ok))
    return log
