"""Adversarial test co-evolution inside RL training, throttled and bounded.

Every ``every`` accepted (correct) candidates of an (operation, dtype) pair,
the hook runs one small co-evolution round (:func:`coevolve_tests`) against
the accepted kernel. Genomes whose error exceeds the task's tolerance are
stored in a per-(operation, dtype) registry (JSON on disk, capped size) and
replayed as extra correctness cases for every later candidate of that pair,
so a test that broke one kernel keeps guarding the others. A wall-clock
budget per round keeps the hook from stalling the training step.
Reference parity: kore/verify/adversarial_hook.py:371-625.
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import asdict
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from .adversarial import Genome, coevolve_tests


class AdversarialRegistry:
    def __init__(self, path: Optional[str] = None, cap: int = 32):
        self.path, self.cap = path, cap
        self.items: Dict[str, List[dict]] = {}
        if path and os.path.exists(path):
            self.items = json.load(open(path))

    @staticmethod
    def key(operation: str, dtype: str) -> str:
        return f"{operation}|{dtype}"

    def add(self, operation: str, dtype: str, genome: Genome, err: float) -> None:
        lst = self.items.setdefault(self.key(operation, dtype), [])
        lst.append(dict(asdict(genome), err=float(min(err, 1e30))))
        lst.sort(key=lambda d: -d["err"])
        del lst[self.cap:]
        if self.path:
            tmp = self.path + ".tmp"
            json.dump(self.items, open(tmp, "w"))
            os.replace(tmp, self.path)

    def genomes(self, operation: str, dtype: str) -> List[Genome]:
        return [Genome(d["regime"], d["scale"], d["sparsity"], d["seed"], d.get("offset", 0.0), d.get("slot", -1))
                for d in self.items.get(self.key(operation, dtype), [])]


def rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    o, r = out.float(), ref.float()
    if not torch.isfinite(o).all() and torch.isfinite(r).all():
        return float("inf")
    return float((o - r).norm() / (r.norm() + 1e-12))


class AdversarialHook:
    def __init__(self, registry: AdversarialRegistry, every: int = 8, budget_s: float = 5.0, tol: float = 2e-2,
                 population: int = 6, generations: int = 2, clock: Callable[[], float] = time.time):
        self.reg, self.every, self.budget_s, self.tol = registry, every, budget_s, tol
        self.population, self.generations, self.clock = population, generations, clock
        self.accepted: Dict[str, int] = {}
        self.rounds = 0

    def replay(self, operation: str, dtype: str, make_inputs: Callable[[int], Sequence[torch.Tensor]],
               candidate: Callable, oracle: Callable) -> Tuple[bool, Optional[str]]:
        """Run the registry's genomes against a candidate: (passed, failing regime)."""
        for g in self.reg.genomes(operation, dtype):
            ins = g.inputs(tuple(make_inputs(g.seed)))
            try:
                if rel_err(candidate(*ins), oracle(*ins)) > self.tol:
                    return False, g.regime
            except Exception:  # noqa: BLE001 - a crash on a registered input is a failure
                return False, g.regime
        return True, None

    def on_accepted(self, operation: str, dtype: str, make_inputs, candidate, oracle) -> int:
        """Count an accepted kernel; every ``every``-th one triggers a bounded round.
        Returns the number of new registry entries."""
        k = AdversarialRegistry.key(operation, dtype)
        self.accepted[k] = self.accepted.get(k, 0) + 1
        if self.accepted[k] % self.every:
            return 0
        t0 = self.clock()
        self.rounds += 1
        pop = coevolve_tests(make_inputs, candidate, oracle, rel_err, population=self.population,
                             generations=self.generations, seed=self.rounds)
        added = 0
        for g, err in pop:
            if self.clock() - t0 > self.budget_s:
                break
            if err > self.tol:
                self.reg.add(operation, dtype, g, err)
                added += 1
        return added
