"""Replay cache of verifier observations (JSONL).

Key = sha256(task_id || 0 || source); entries are ``{key, task_id, obs}``;
unknown observation fields from older schemas are dropped on load, so the
cache survives schema drift (reference: kore/env/replay.py:15-72)."""
from __future__ import annotations

import hashlib
import json
import os
import threading
from dataclasses import asdict, fields
from typing import Dict, Optional

from ..reward.reward import Observation


def cache_key(task_id: str, source: str) -> str:
    return hashlib.sha256(f"{task_id}\x00{source}".encode()).hexdigest()


class ReplayCache:
    def __init__(self, path: Optional[str] = None):
        self.path = path
        self.mem: Dict[str, Observation] = {}
        self.lock = threading.Lock()
        if path and os.path.exists(path):
            names = {f.name for f in fields(Observation)}
            with open(path) as f:
                for line in f:
                    try:
                        rec = json.loads(line)
                        self.mem[rec["key"]] = Observation(**{k: v for k, v in rec["obs"].items() if k in names})
                    except (ValueError, KeyError, TypeError):
                        continue

    def get(self, task_id: str, source: str) -> Optional[Observation]:
        return self.mem.get(cache_key(task_id, source))

    def put(self, task_id: str, source: str, obs: Observation) -> None:
        if obs.infra_error:
            return                              # infrastructure failures are never cached
        k = cache_key(task_id, source)
        with self.lock:
            self.mem[k] = obs
            if self.path:
                os.makedirs(os.path.dirname(os.path.abspath(self.path)), exist_ok=True)
                with open(self.path, "a") as f:
                    f.write(json.dumps({"key": k, "task_id": task_id, "obs": asdict(obs)}) + "\n")
