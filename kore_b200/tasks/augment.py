"""Shape augmentation for verification: more shapes per task, so a kernel
that only works for the declared shapes (a hard-coded tile count, no
boundary masks, a specialised power-of-two path) fails verification.

From the task's primary shape it derives, deterministically:

* scaled shapes: the row-like dimension (the first of M, T, rows, B, S that the
  task has) times 1/2 and 2, kept on a multiple of 8;
* one odd shape: that dimension made non-aligned (a multiple of 8 plus 3), the
  case that catches missing edge masks.

Only row-like dimensions change: head counts, head dims, hidden sizes and
vocabularies keep the values the operator's definition expects. Shapes whose
compulsory bytes (roofline model) exceed ``max_bytes`` are skipped, so
augmentation never asks for more memory than the declared shapes by much.
Opt-in through ``KoreConfig.shape_augment`` (``KORE_SHAPE_AUGMENT=1``): the
environment then verifies correctness on these shapes too (the driver takes
them with ``--dims``). Reference parity: kore/tasks/augment.py (scaled plus
one non-aligned shape per base shape), restricted to row-like dims.
"""
from __future__ import annotations

from typing import Dict, List, Optional

from .base import Shape

ROW_DIMS = ("M", "T", "rows", "B", "S")


def row_dim(dims: Dict[str, int]) -> Optional[str]:
    for k in ROW_DIMS:
        if isinstance(dims.get(k), int) and dims[k] >= 8:
            return k
    return None


def _round8(v: float) -> int:
    return max(8, int(round(v / 8.0)) * 8)


def augment_shapes(task, max_n: int = 6, max_bytes: float = 4e9) -> List[Shape]:
    prim = task.shape("primary") or (task.shapes[0] if task.shapes else None)
    if prim is None:
        return []
    k = row_dim(prim.dims)
    if k is None:
        return []
    base = prim.dims[k]
    cands = [_round8(base * 0.5), _round8(base * 2), _round8(base * 0.5) + 3]
    from ..analysis.rooflines import flops_bytes
    out: List[Shape] = []
    seen = {base}
    for i, v in enumerate(cands):
        if v in seen or v < 1:
            continue
        seen.add(v)
        dims = dict(prim.dims)
        dims[k] = v
        fb = flops_bytes(task.operation, dims, task.dtype)
        if fb is not None and fb[1] > max_bytes:
            continue
        out.append(Shape(f"aug{i}_{k}{v}", dims))
        if len(out) >= max_n:
            break
    return out
