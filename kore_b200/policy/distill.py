"""Distillation sink for the co-evolution loop: keeps, per (task, kernel
source), the best verified speedup and writes them as ``WinRecord`` JSONL
(deduplicated by sha256 of task id and source), so winning kernels found
during GRPO / search feed the next SFT round.
Reference parity: kore/policy/coevolve_distill.py:87-230.
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Dict, List, Optional

from ..data.schemas import WinRecord, read_records


def _key(task_id: str, src: str) -> str:
    return hashlib.sha256(f"{task_id}\0{src}".encode()).hexdigest()


class DistillSink:
    def __init__(self, path: Optional[str] = None, min_speedup: float = 1.0):
        self.path, self.min_speedup = path, min_speedup
        self.best: Dict[str, WinRecord] = {}
        if path and os.path.exists(path):
            for r in read_records(path, WinRecord):
                k = _key(r.task_id, r.final_kernel or "")
                if k not in self.best or (r.speedup or 0) > (self.best[k].speedup or 0):
                    self.best[k] = r

    def add(self, task_id: str, src: str, speedup: float, messages: Optional[List[dict]] = None,
            operation: Optional[str] = None, baseline_us: Optional[float] = None) -> bool:
        if speedup is None or speedup <= self.min_speedup:
            return False
        k = _key(task_id, src)
        cur = self.best.get(k)
        if cur is not None and (cur.speedup or 0) >= speedup:
            return False
        self.best[k] = WinRecord(task_id=task_id, trajectory=messages or [], initial_wall_us=baseline_us,
                                 final_wall_us=(baseline_us / speedup) if baseline_us else None, speedup=speedup,
                                 operation=operation, final_kernel=src)
        return True

    def flush(self) -> int:
        if not self.path:
            return 0
        tmp = self.path + ".tmp"
        with open(tmp, "w") as f:
            for r in sorted(self.best.values(), key=lambda r: (r.task_id, -(r.speedup or 0))):
                f.write(json.dumps(r.to_dict()) + "\n")
        os.replace(tmp, self.path)
        return len(self.best)
