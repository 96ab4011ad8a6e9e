"""Measurement allocation for the search: a hard verifier-call budget,
streaming statistics with a pessimistic lower confidence bound, and
successive halving.

The search ranks and commits by the LCB of a kernel's measured speedup, not
its mean: a fast but noisy kernel must not beat a slightly slower stable one.
An arm with one sample has an LCB of ``mean - single_sample_penalty`` (its
spread is unknown), none has minus infinity.

Reference behaviour: kore/search/bandit.py:49-258 (Budget, streaming
mean/variance with LCB, SHA rung schedule).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, Hashable, List, Optional, Sequence


@dataclass
class Budget:
    """Hard cap on verifier (environment) calls."""

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

    def exhausted(self) -> bool:
        return self.used >= self.total


@dataclass
class MeasureStats:
    """Welford mean / variance of the samples of one arm."""

    n: int = 0
    mean: float = 0.0
    m2: float = 0.0
    single_sample_penalty: float = 0.1

    def add(self, x: float) -> None:
        self.n += 1
        d = x - self.mean
        self.mean += d / self.n
        self.m2 += d * (x - self.mean)

    def var(self) -> float:
        return self.m2 / (self.n - 1) if self.n > 1 else math.inf

    def stderr(self) -> float:
        return math.sqrt(self.var() / self.n) if self.n > 1 else math.inf

    def lcb(self, z: float = 1.0) -> float:
        if self.n == 0:
            return -math.inf
        if self.n == 1:
            return self.mean - self.single_sample_penalty * abs(self.mean)
        return self.mean - z * self.stderr()

    def ucb(self, z: float = 1.0) -> float:
        if self.n < 2:
            return math.inf
        return self.mean + z * self.stderr()


ArmStats = MeasureStats     # name kept for earlier callers


def rung_schedule(n_arms: int, budget: int, eta: int = 2, min_pulls: int = 1) -> List[int]:
    """Pulls per surviving arm at each rung of successive halving, sized so
    the whole schedule fits ``budget``."""
    rungs, alive, pulls, spent = [], n_arms, min_pulls, 0
    while alive >= 1 and spent + alive * pulls <= budget:
        rungs.append(pulls)
        spent += alive * pulls
        if alive == 1:
            break
        alive = max(1, alive // eta)
        pulls *= eta
    return rungs


def successive_halving(arms: Sequence[Hashable], evaluate: Callable[[Hashable], float], budget: Budget,
                       eta: int = 2, z: float = 1.0, min_pulls: int = 1,
                       stats: Optional[Dict[Hashable, MeasureStats]] = None) -> Hashable:
    """Pull every survivor, keep the top 1/eta by LCB, repeat with eta x the
    pulls while the budget lasts; return the survivor with the best LCB
    (mean as tie-break)."""
    stats = stats if stats is not None else {}
    for a in arms:
        stats.setdefault(a, MeasureStats())
    alive: List[Hashable] = list(arms)
    pulls = min_pulls
    while alive:
        if budget.left < len(alive):
            break
        for a in alive:
            for _ in range(pulls):
                if not budget.take():
                    break
                stats[a].add(float(evaluate(a)))
        alive.sort(key=lambda a: (stats[a].lcb(z), stats[a].mean), reverse=True)
        if len(alive) == 1:
            break
        alive = alive[: max(1, len(alive) // eta)]
        pulls *= eta
    pool = alive or list(arms)
    return max(pool, key=lambda a: (stats[a].lcb(z), stats[a].mean if stats[a].n else -math.inf))
