"""Data-scale audit of the task corpus, computed from the live registry (so
it cannot drift from the tasks that exist): operators, families, dtypes,
operation classes, the train / held-out split, declared shapes and the shapes
verification sees with augmentation on, and how many tasks have a roofline.

    python -m kore_b200.tasks.audit [--json]   (also: kore tasks --audit)

Reference parity: kore/tasks/audit.py (DataScaleReport from the registry,
including shape augmentation).
"""
from __future__ import annotations

import argparse
import json
from collections import Counter
from dataclasses import asdict, dataclass
from typing import Dict


@dataclass
class DataScaleReport:
    tasks: int
    train: int
    heldout: int
    families: Dict[str, int]
    dtypes: Dict[str, int]
    op_classes: Dict[str, int]
    declared_shapes: int
    augmented_shapes: int
    with_roofline: int
    external: int = 0            # problems registered at run time without an operation model (KernelBench)

    def as_dict(self) -> dict:
        return asdict(self)

    def render(self) -> str:
        top = ", ".join(f"{k} {v}" for k, v in sorted(self.families.items(), key=lambda kv: -kv[1])[:12])
        return (f"{self.tasks} tasks ({self.train} train / {self.heldout} held out); "
                f"{len(self.families)} families ({top}); dtypes {self.dtypes}; operation classes {self.op_classes}; "
                f"{self.declared_shapes} declared shapes, {self.augmented_shapes} more with augmentation; "
                f"{self.with_roofline} tasks with a roofline")


def audit(augment_max: int = 6) -> DataScaleReport:
    from ..analysis.rooflines import flops_bytes
    from ..value.features import op_class
    from .augment import augment_shapes
    from .registry import all_tasks, split_tasks
    ts = all_tasks()
    tr, ho = split_tasks()
    fam, dt, oc = Counter(), Counter(), Counter()
    shapes = aug = roof = ext = 0
    for t in ts:
        if t.operation == "kernelbench":
            ext += 1
        fam[t.family] += 1
        dt[t.dtype] += 1
        oc[op_class(t.operation)] += 1
        shapes += len(t.shapes)
        aug += len(augment_shapes(t, augment_max))
        sh = t.shape("primary") or (t.shapes[0] if t.shapes else None)
        if sh is not None and flops_bytes(t.operation, sh.dims, t.dtype) is not None:
            roof += 1
    return DataScaleReport(len(ts), len(tr), len(ho), dict(fam), dict(dt), dict(oc), shapes, aug, roof, ext)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore tasks --audit")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    r = audit()
    print(json.dumps(r.as_dict(), indent=1) if a.json else r.render())
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
