"""The open-ended generation loop (POET-shaped): propose tasks at the
frontier, attempt them with the current policy, record outcomes, distill
wins, and periodically grow the task space by minting.

``attempt(task_id) -> (solve_rate or success, best_speedup)``;
``distill(task_id, speedup)`` receives verified wins above 1x.
Reference behaviour: kore/openended/coevolve.py:82-174.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Tuple

from .controller import CoevolutionController


def coevolve(controller: CoevolutionController, attempt: Callable[[str], Tuple[float, float]], rounds: int = 4,
             batch: int = 4, distill: Optional[Callable[[str, float], None]] = None,
             mint_every: int = 0) -> List[Tuple[str, bool]]:
    log: List[Tuple[str, bool]] = []
    for r in range(rounds):
        if mint_every and r and r % mint_every == 0:
            controller._mint(controller._rng())
        for tid in controller.next_task_id(batch):
            ok, speed = attempt(tid)
            rate = float(ok)
            controller.record(tid, rate, speedup=speed if rate > 0 else None,
                              regret=max(0.0, 1.0 - speed) if rate > 0 else 1.0)
            if rate > 0 and distill is not None and speed > 1.0:
                distill(tid, speed)
            log.append((tid, bool(rate > 0)))
    return log


def frontier_report(controller: CoevolutionController) -> Dict[str, object]:
    a = controller.archive
    tried = [e for e in a.entries.values() if e.attempts]
    return {"tasks": len(a.entries), "niches": len(a.cells), "coverage": round(a.coverage(), 4),
            "attempted": len(tried), "minted": len(controller.minted),
            "mean_p": round(sum(e.p for e in tried) / max(1, len(tried)), 4),
            "frontier": [e.desc.task_id for e in a.elites()[:5]]}
