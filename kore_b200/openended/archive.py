"""MAP-Elites archive of curriculum tasks.

Per task, :class:`DescriptorStats` keeps what the curriculum learned about
it: attempts, a solve-rate estimate (Beta(1,1) prior, exponentially
discounted so a task the policy has since mastered stops looking hard), the
best verified speedup and the headroom regret (unrealised speedup against
the roofline, in [0, 1]). Per niche (behaviour cell) the archive keeps the
elite: the task whose frontier score is highest, so the proposer sees one
representative per region of the behaviour space plus everything it has
evidence about.

Reference behaviour: kore/openended/archive.py:28-149.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

from .task_space import TaskDescriptor


@dataclass
class DescriptorStats:
    desc: TaskDescriptor
    attempts: int = 0
    succ_w: float = 0.0          # discounted successes
    tot_w: float = 0.0           # discounted attempts
    best_speedup: float = 0.0
    regret: float = 1.0          # unrealised headroom in [0, 1]; 1 = nothing achieved yet
    discount: float = 0.95

    @property
    def p(self) -> float:
        return (self.succ_w + 1.0) / (self.tot_w + 2.0)

    @property
    def has_evidence(self) -> bool:
        return self.attempts > 0

    @property
    def successes(self) -> int:              # earlier field name
        return int(round(self.succ_w))

    @property
    def informativeness(self) -> float:
        return 4.0 * self.p * (1.0 - self.p)

    def observe(self, solve_rate: float, speedup: Optional[float] = None, ceiling: Optional[float] = None) -> None:
        self.attempts += 1
        self.succ_w = self.discount * self.succ_w + float(solve_rate)
        self.tot_w = self.discount * self.tot_w + 1.0
        if speedup is not None and speedup > self.best_speedup:
            self.best_speedup = float(speedup)
        if ceiling and ceiling > 0:
            self.regret = max(0.0, min(1.0, 1.0 - self.best_speedup / ceiling))
        elif speedup is not None:
            self.regret = max(0.0, min(1.0, 1.0 - min(self.best_speedup, 2.0) / 2.0))


ArchiveEntry = DescriptorStats      # earlier name


class TaskArchive:
    def __init__(self):
        self.entries: Dict[str, DescriptorStats] = {}
        self.cells: Dict[Tuple, DescriptorStats] = {}

    def add(self, d: TaskDescriptor) -> DescriptorStats:
        e = self.entries.get(d.task_id)
        if e is None:
            e = self.entries[d.task_id] = DescriptorStats(d)
        self._place(e, lambda x: x.informativeness)
        return e

    def _place(self, e: DescriptorStats, score: Callable[[DescriptorStats], float]) -> None:
        cell = e.desc.niche()
        cur = self.cells.get(cell)
        if cur is None or cur is e or score(e) > score(cur):
            self.cells[cell] = e

    def record(self, tid: str, success, regret: Optional[float] = None, speedup: Optional[float] = None,
               ceiling: Optional[float] = None,
               score: Optional[Callable[[DescriptorStats], float]] = None) -> DescriptorStats:
        e = self.entries[tid]
        e.observe(float(success), speedup, ceiling)
        if regret is not None:
            e.regret = max(0.0, min(1.0, float(regret)))
        self._place(e, score or (lambda x: x.informativeness + 0.5 * x.regret))
        return e

    def occupied(self) -> List[Tuple]:
        return [c for c, e in self.cells.items() if e.has_evidence]

    def elites(self) -> List[DescriptorStats]:
        return sorted(self.cells.values(), key=lambda e: (-(e.informativeness + 0.5 * e.regret), e.desc.task_id))

    def coverage(self) -> float:
        return len(self.occupied()) / max(1, len(self.cells))
