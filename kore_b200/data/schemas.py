"""Typed records of the data factory, stored as JSONL.

* ``RepairRecord``: a failing parent kernel (compile / SNR failure) and the
  teacher's repair, as chat messages (SFT, repair-weighted).
* ``RankedGroupRecord``: a parent and k candidates ranked by verified
  speed; preference pairs (chosen, rejected) for DPO.
* ``WinRecord``: a full multi-turn trajectory that improved wall time.
Field names match the reference's JSONL format (kore/data/schemas.py:29-218)
so existing datasets load unchanged; ``gpu`` defaults to "b200".
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path
from typing import Iterable, Iterator, List, Optional, Type, TypeVar

GPU_DEFAULT = "b200"
T = TypeVar("T")


def _from(cls, d: dict):
    names = {f.name for f in fields(cls)}
    return cls(**{k: v for k, v in d.items() if k in names})


@dataclass
class RepairRecord:
    task_id: str
    failure_class: str
    parent_hash: str
    error_text: str
    messages: List[dict]
    child_snr_db: Optional[float] = None
    type: str = "repair"
    operator: str = "repair"
    gpu: str = GPU_DEFAULT
    operation: Optional[str] = None
    arch: Optional[str] = None
    shape: Optional[str] = None

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "RepairRecord":
        return _from(cls, d)


@dataclass
class RankedGroupRecord:
    task_id: str
    parent_id: str
    candidates: List[dict]
    preferences: List[List[int]]
    type: str = "ranked_group"
    gpu: str = GPU_DEFAULT
    operation: Optional[str] = None
    arch: Optional[str] = None
    shape: Optional[str] = None
    counters: Optional[dict] = None
    parent_counters: Optional[dict] = None
    parent_wall_us: Optional[float] = None

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "RankedGroupRecord":
        return _from(cls, d)


@dataclass
class WinRecord:
    task_id: str
    trajectory: List[dict]
    initial_wall_us: Optional[float]
    final_wall_us: Optional[float]
    speedup: Optional[float]
    type: str = "win"
    gpu: str = GPU_DEFAULT
    operation: Optional[str] = None
    arch: Optional[str] = None
    shape: Optional[str] = None
    final_kernel: Optional[str] = None

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "WinRecord":
        return _from(cls, d)


_TYPES = {"repair": RepairRecord, "ranked_group": RankedGroupRecord, "win": WinRecord}


def write_records(path, records: Iterable) -> int:
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    n = 0
    with open(path, "a") as f:
        for r in records:
            f.write(json.dumps(r.to_dict()) + "\n")
            n += 1
    return n


def read_records(path, cls: Optional[Type[T]] = None) -> Iterator:
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                d = json.loads(line)
            except json.JSONDecodeError:
                continue
            k = cls or _TYPES.get(d.get("type", ""), None)
            if k is not None:
                yield k.from_dict(d)
