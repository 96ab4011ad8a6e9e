"""Task ABI: a task binds an operator spec to named shapes.

On disk a task is a directory with ``task.yaml`` (``task_id``, ``operation``,
``dtype``, ``backend``, ``gpu_target``, ``seed_kernel_name``,
``snr_threshold``, ``shapes{minimal, primary, validation[]}``, ``targets``)
plus optional ``reference.py`` / seed kernel; library tasks are built from
:mod:`kore_b200.tasks.ops_library` specs. Reference parity:
kore/tasks/base.py:24-96 (Task / Shape / from_dir).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class Shape:
    name: str
    dims: Dict[str, int]

    def as_args(self) -> str:
        return ",".join(f"{k}={v}" for k, v in self.dims.items())


@dataclass
class Task:
    task_id: str
    operation: str
    dtype: str = "bf16"
    backend: str = "triton"
    gpu_target: str = "sm_100a"
    entry: str = ""
    spec: str = ""                       # ops_library spec name
    snr_threshold: Optional[float] = None
    shapes: List[Shape] = field(default_factory=list)
    seed_src: str = ""
    reference_src: str = ""
    targets: dict = field(default_factory=dict)
    family: str = "core"
    path: Optional[str] = None

    def shape(self, name: str) -> Optional[Shape]:
        for s in self.shapes:
            if s.name == name:
                return s
        return None

    @property
    def shapes_text(self) -> str:
        return "; ".join(f"{s.name}: {s.as_args()}" for s in self.shapes)

    def bench_shapes(self) -> List[Shape]:
        return [s for s in self.shapes if s.name != "minimal"]

    @staticmethod
    def from_spec(spec) -> "Task":
        shapes = []
        sh = spec.shapes
        if "minimal" in sh:
            shapes.append(Shape("minimal", dict(sh["minimal"])))
        if "primary" in sh:
            shapes.append(Shape("primary", dict(sh["primary"])))
        for i, d in enumerate(sh.get("validation", []) or []):
            shapes.append(Shape(f"validation{i}", dict(d)))
        import inspect
        try:
            ref_src = inspect.getsource(spec.reference)
        except (OSError, TypeError):
            ref_src = ""
        return Task(task_id=spec.name, operation=spec.operation, dtype=spec.dtype, entry=spec.entry,
                    spec=spec.name, snr_threshold=spec.snr_threshold, shapes=shapes, seed_src=spec.seed_src,
                    reference_src=ref_src, family=spec.family,
                    targets={"comparison_baseline": "vendor (cuBLAS / cuDNN / torch fused)"})

    @staticmethod
    def from_dir(path: str) -> "Task":
        import yaml
        with open(os.path.join(path, "task.yaml")) as f:
            y = yaml.safe_load(f)
        shapes = []
        sh = y.get("shapes", {}) or {}
        for k in ("minimal", "primary"):
            if k in sh:
                shapes.append(Shape(k, dict(sh[k])))
        for i, d in enumerate(sh.get("validation", []) or []):
            shapes.append(Shape(f"validation{i}", dict(d)))
        seed_name = y.get("seed_kernel_name", "seed_kernel.py")
        seed = open(os.path.join(path, seed_name)).read() if os.path.exists(os.path.join(path, seed_name)) else ""
        ref_p = os.path.join(path, "reference.py")
        return Task(task_id=y["task_id"], operation=y.get("operation", ""), dtype=y.get("dtype", "bf16"),
                    backend=y.get("backend", "triton"), gpu_target=y.get("gpu_target", "sm_100a"),
                    entry=y.get("entry", ""), spec=y.get("spec", ""), snr_threshold=y.get("snr_threshold"),
                    shapes=shapes, seed_src=seed,
                    reference_src=open(ref_p).read() if os.path.exists(ref_p) else "",
                    targets=y.get("targets", {}) or {}, family=y.get("family", "core"), path=path)
