"""Parametric task space of the open-ended curriculum.

A :class:`TaskDescriptor` places a kernel task in a behaviour space:
family, operation, dtype, shape regime (log2 size bucket), arithmetic
intensity bucket, and fusion depth (how many primitive ops a fused task
chains). The MAP-Elites archive uses ``niche()`` (the discretised
behaviour) and the proposer's novelty is the Hamming distance between
niches.

Held-out safety: descriptors are built only from the trainer's registry with
the held-out families filtered out (``HELD_OUT_FAMILIES``), so the curriculum
cannot represent, and hence never proposes, a held-out task.

``mutate`` moves a descriptor to a neighbouring point (other dtype, shape
one regime up or down, sibling operation of the same family); the controller
maps a mutated descriptor back to the closest registered task.

Reference behaviour: kore/openended/task_space.py:111-363.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, replace
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

HELD_OUT_FAMILIES = ("mla", "paged_attention", "held_out")
PRECISION = {"fp32": 0, "tf32": 1, "fp16": 2, "bf16": 2, "fp8": 3, "fp8_e4m3": 3, "fp8_e5m2": 3, "int8": 3,
             "mxfp4": 4, "fp4": 4}


@dataclass(frozen=True)
class TaskDescriptor:
    task_id: str
    family: str
    operation: str
    dtype: str
    dims: Tuple[Tuple[str, int], ...] = ()
    fusion_depth: int = 1

    @property
    def size(self) -> int:
        n = 1
        for _, v in self.dims:
            n *= max(1, int(v))
        return n

    def scale(self) -> int:
        """Shape regime: log2 of the element count in buckets of 4 (x16)."""
        return int(math.log2(max(1, self.size))) // 4

    def intensity(self) -> float:
        from ..analysis.rooflines import flops_bytes
        fb = flops_bytes(self.operation, dict(self.dims), self.dtype)
        return fb[0] / fb[1] if fb and fb[1] else 0.0

    def niche(self) -> Tuple[str, int, int, int, int]:
        return (self.family, int(math.log2(1.0 + self.intensity())), min(self.fusion_depth, 4),
                PRECISION.get(self.dtype, 1), self.scale())

    def features(self) -> Tuple[str, int, int, int, int]:      # earlier name
        return self.niche()


def niche_distance(a: Sequence, b: Sequence) -> int:
    return sum(1 for x, y in zip(a, b) if x != y)


def _fusion_depth(task) -> int:
    tid = getattr(task, "task_id", "")
    if tid.startswith("minted_"):
        return max(1, tid.count("(") or tid.count("_") // 2)
    op = (getattr(task, "operation", "") or "").lower()
    return 1 + sum(1 for k in ("fused", "residual", "bias", "gelu", "silu", "norm", "+") if k in op)


def descriptor_of(task) -> Optional[TaskDescriptor]:
    if getattr(task, "family", "") in HELD_OUT_FAMILIES:
        return None
    sh = task.shape("primary") if hasattr(task, "shape") else None
    sh = sh or (task.shapes[0] if getattr(task, "shapes", None) else None)
    if sh is None:
        return None
    return TaskDescriptor(task.task_id, task.family or "misc", task.operation, task.dtype,
                          tuple(sorted((k, int(v)) for k, v in sh.dims.items() if isinstance(v, int))),
                          _fusion_depth(task))


class TaskSpace:
    """The descriptors of the trainable tasks (optionally restricted to an
    allowed list), indexed by id and niche."""

    def __init__(self, tasks: Optional[Iterable] = None, allowed: Optional[Iterable[str]] = None):
        if tasks is None:
            from ..tasks.registry import all_tasks
            tasks = all_tasks()
        allow = set(allowed) if allowed is not None else None
        self.items: List[TaskDescriptor] = []
        for t in tasks:
            if allow is not None and t.task_id not in allow:
                continue
            d = descriptor_of(t)
            if d is not None:
                self.items.append(d)
        self._by_id: Dict[str, TaskDescriptor] = {d.task_id: d for d in self.items}

    def __len__(self) -> int:
        return len(self.items)

    def by_id(self, tid: str) -> Optional[TaskDescriptor]:
        return self._by_id.get(tid)

    def add(self, d: TaskDescriptor) -> None:
        if d.family in HELD_OUT_FAMILIES or d.task_id in self._by_id:
            return
        self.items.append(d)
        self._by_id[d.task_id] = d

    def nearest(self, d: TaskDescriptor, exclude: Sequence[str] = ()) -> Optional[TaskDescriptor]:
        """The registered descriptor closest to ``d`` (niche distance, then size)."""
        ex = set(exclude)
        cand = [x for x in self.items if x.task_id not in ex]
        if not cand:
            return None
        n = d.niche()
        return min(cand, key=lambda x: (niche_distance(x.niche(), n), abs(math.log2(max(1, x.size)) -
                                                                       math.log2(max(1, d.size))), x.task_id))

    def mutate(self, d: TaskDescriptor, rng: random.Random) -> TaskDescriptor:
        """A neighbouring point of the space (not necessarily registered)."""
        kind = rng.choice(("dtype", "scale", "sibling"))
        if kind == "dtype":
            options = sorted({x.dtype for x in self.items if x.operation == d.operation} - {d.dtype}) or \
                sorted({x.dtype for x in self.items} - {d.dtype})
            return replace(d, dtype=rng.choice(options)) if options else d
        if kind == "scale":
            f = 2 if rng.random() < 0.5 else 0.5
            dims = tuple((k, max(1, int(v * f))) for k, v in d.dims)
            return replace(d, dims=dims)
        sib = sorted({x.operation for x in self.items if x.family == d.family} - {d.operation})
        return replace(d, operation=rng.choice(sib)) if sib else d
