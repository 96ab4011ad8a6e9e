"""Evaluation budget, lower-confidence-bound statistics and successive halving
(reference parity: kore/search/bandit.py:49-258)."""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, Hashable, List, Sequence


@dataclass
class Budget:
    total: int
    used: int = 0

    def take(self, n: int = 1) -> bool:
        if self.used + n > self.total:
            return False
        self.used += n
        return True

    @property
    def left(self) -> int:
        return self.total - self.used


@dataclass
class ArmStats:
    n: int = 0
    mean: float = 0.0
    m2: float = 0.0

    def add(self, x: float) -> None:
        self.n += 1
        d = x - self.mean
        self.mean += d / self.n
        self.m2 += d * (x - self.mean)

    def lcb(self, z: float = 1.0) -> float:
        if self.n < 2:
            return -math.inf if self.n == 0 else self.mean - 1.0
        return self.mean - z * math.sqrt(self.m2 / (self.n - 1) / self.n)

    def ucb(self, z: float = 1.0) -> float:
        if self.n < 2:
            return math.inf
        return self.mean + z * math.sqrt(self.m2 / (self.n - 1) / self.n)


def successive_halving(arms: Sequence[Hashable], evaluate: Callable[[Hashable], float], budget: Budget,
                       eta: int = 2, z: float = 1.0) -> Hashable:
    """Evaluate all survivors once per round, keep the top 1/eta by LCB."""
    stats: Dict[Hashable, ArmStats] = {a: ArmStats() for a in arms}
    alive: List[Hashable] = list(arms)
    while len(alive) > 1 and budget.left >= len(alive):
        for a in alive:
            budget.take()
            stats[a].add(evaluate(a))
        alive.sort(key=lambda a: (stats[a].lcb(z), stats[a].mean), reverse=True)
        alive = alive[: max(1, len(alive) // eta)]
    return max(alive, key=lambda a: stats[a].mean)
