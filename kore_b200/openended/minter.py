"""TaskMinter: net-new, correct-by-construction kernel tasks from the typed
grammar, grown beyond the registered menu.

Moves (each proposes a :class:`~kore_b200.openended.grammar.Pipeline`):

* ``fusion``       chain 2-4 primitives into one fused op;
* ``extrapolate``  an existing structure at another dtype or shape scale;
* ``novel``        activations and row reductions composed into a new op;
* ``crossover``    lift two registered operations into the grammar and splice
                   the head of one onto the tail of the other.

Construction gate (every check must pass before a task is registered):
(1) well typed, (2) not a held-out family, (3) runs on CPU, (4) finite,
(5) deterministic for a seed, (6) not constant, (7) varies along every output
axis, (8) sensitive to every input. Survivors are de-duplicated by
(behavioural hash, dtype, shape scale) and registered as library specs whose
reference is the pipeline itself; the seed is the torch reference (the
policy writes the kernel). ``materialize`` writes a registered spec as a task
directory in the task ABI and reloads it as a self-check.

Reference behaviour: kore/openended/minter.py:323-844, materialize.py:232.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Set, Tuple

from ..tasks.spec import OpSpec
from .grammar import MAT, Pipeline, lift, primitives, random_pipeline
from .task_space import HELD_OUT_FAMILIES

MOVES = ("fusion", "extrapolate", "novel", "crossover")
DTYPES = ("bf16", "fp16", "fp32")
SHAPES = ({"M": 4096, "N": 4096}, {"M": 8192, "N": 2048}, {"M": 2048, "N": 8192}, {"M": 16384, "N": 1024})


@dataclass
class MintedTask:
    task_id: str
    pipeline: Pipeline
    dtype: str
    shapes: Dict[str, object]
    move: str
    bhash: str
    family: str = "minted"


def gate_pipeline(p: Pipeline, family: str = "minted", dims=(16, 32)) -> Optional[str]:
    """The eight construction checks; None when the pipeline passes."""
    import torch
    why = p.typecheck()
    if why:
        return "ill-typed: " + why
    if any(h in family.lower() or h in p.name for h in HELD_OUT_FAMILIES):
        return "held-out family"
    M, N = dims
    sample, ref = p.build_sampler(), p.build_reference()
    try:
        ins = sample({"M": M, "N": N}, 7, "cpu", torch.float32)
        y = ref(*ins)
    except Exception as e:  # noqa: BLE001
        return f"raises {type(e).__name__}"
    if not torch.isfinite(y).all():
        return "non-finite"
    if not torch.equal(y, ref(*sample({"M": M, "N": N}, 7, "cpu", torch.float32))):
        return "non-deterministic"
    tol = 1e-5 * max(1.0, float(y.abs().max()))
    if float(y.max() - y.min()) <= tol:
        return "constant output"
    for ax in range(y.dim()):
        if y.shape[ax] > 1 and float(y.std(dim=ax).max()) <= tol:
            return f"constant along axis {ax}"
    for i, t in enumerate(ins):
        bumped = list(ins)
        bumped[i] = t + 0.5 * torch.randn_like(t)
        if torch.allclose(ref(*bumped), y, atol=1e-6):
            return f"ignores input {i}"
    return None


def construction_gate(fn: Callable, dims=(64, 256)) -> Optional[str]:
    """The gate for a plain two-input function f(a, b) (same shape in and out)."""
    import torch
    a, b = torch.randn(*dims), torch.randn(*dims)
    try:
        y = fn(a, b)
    except Exception as e:  # noqa: BLE001
        return f"raises {type(e).__name__}"
    if y.shape != a.shape:
        return "shape changes"
    if not torch.isfinite(y).all():
        return "non-finite"
    if not torch.equal(y, fn(a, b)):
        return "non-deterministic"
    if torch.allclose(fn(a + 1.0, b), y):
        return "ignores input a"
    if torch.allclose(fn(a, b + 1.0), y):
        return "ignores input b"
    if float(y.abs().max()) == 0.0:
        return "trivial output"
    return None


def _seed_source(task_id: str, p: Pipeline, n_aux: int) -> str:
    args = ", ".join(["x"] + [f"a{i}" for i in range(n_aux)])
    return ("import torch\n\n\n"
            f"def fused({args}):\n"
            f"    \"\"\"{' -> '.join(p.stages)} (reference composition; write the fused kernel).\"\"\"\n"
            f"    raise NotImplementedError('{task_id}')\n")


class TaskMinter:
    def __init__(self, seed: int = 0, registry: Optional[Dict[str, OpSpec]] = None):
        self.rng = random.Random(seed)
        if registry is None:
            from ..tasks.ops_library import SPECS
            registry = SPECS
        self.registry = registry
        self.seen: Set[Tuple[str, str, int]] = set()
        self.rejected: Dict[str, int] = {}
        self.minted: List[MintedTask] = []

    # ------------------------------------------------------------------ moves
    def _propose(self, move: str) -> Tuple[Pipeline, str, Dict[str, int]]:
        rng = self.rng
        shape = dict(rng.choice(SHAPES))
        dtype = rng.choice(DTYPES[:2])
        if move == "fusion":
            p = random_pipeline(rng, rng.randint(2, 4), terminal=False)
        elif move == "novel":
            p = random_pipeline(rng, rng.randint(2, 3), allow_matmul=False, terminal=True)
        elif move == "extrapolate" and self.minted:
            base = rng.choice(self.minted)
            p = Pipeline(list(base.pipeline.stages), base.pipeline.width_out)
            dtype = rng.choice([d for d in DTYPES if d != base.dtype])
            shape = {k: max(256, v * rng.choice((2, 1)) // rng.choice((1, 2))) for k, v in base.shapes["primary"].items()}
        else:                                   # crossover of lifted registered operations
            lifted = [q for q in (lift(s.operation) or lift(s.name) for s in self.registry.values()) if q]
            if len(lifted) >= 2:
                a, b = rng.sample(lifted, 2)
                cut_a, cut_b = rng.randint(1, len(a.stages)), rng.randint(0, len(b.stages) - 1)
                p = Pipeline(a.stages[:cut_a] + b.stages[cut_b:])
            else:
                p = random_pipeline(rng, 3)
            move = "crossover"
        if "matmul" in p.stages:
            p.width_out = rng.choice((shape["N"], shape["N"] // 2, shape["N"] * 2))
        return p, dtype, shape

    # ------------------------------------------------------------------ mint
    def mint(self, n: int = 4, max_tries: Optional[int] = None, moves: Sequence[str] = MOVES) -> List[str]:
        made: List[str] = []
        tries = 0
        while len(made) < n and tries < (max_tries or 60 * n):
            tries += 1
            move = moves[tries % len(moves)]
            p, dtype, shape = self._propose(move)
            why = gate_pipeline(p)
            if why:
                key = why.split(":")[0].split(" ")[0]
                self.rejected[key] = self.rejected.get(key, 0) + 1
                continue
            bh = p.behavioral_hash()
            scale = (shape["M"] * shape["N"]).bit_length() // 4
            if (bh, dtype, scale) in self.seen:
                self.rejected["duplicate"] = self.rejected.get("duplicate", 0) + 1
                continue
            self.seen.add((bh, dtype, scale))
            tid = f"minted_{p.name}_{dtype}_{bh[:6]}"[:80]
            if tid in self.registry:
                continue
            shapes = {"minimal": {"M": 64, "N": 256}, "primary": dict(shape), "validation": []}
            if "matmul" in p.stages:
                shapes["primary"]["N_out"] = p.width_out or shape["N"]
            mt = MintedTask(tid, p, dtype, shapes,
                            move, bh)
            self._register(mt)
            self.minted.append(mt)
            made.append(tid)
        return made

    def _register(self, mt: MintedTask) -> None:
        p = mt.pipeline
        ref = p.build_reference()
        sample = p.build_sampler()
        n_aux = len(p.aux_specs(1, 1))
        op = "gemm_fused" if "matmul" in p.stages else ("reduce_fused" if p.out_type != MAT else "elementwise_fused")

        def reference(*x, ref=ref):
            return ref(*[t.float() for t in x]).float()

        def baseline(*x, ref=ref):
            import torch
            with torch.no_grad():
                return ref(*x).to(x[0].dtype)
        self.registry[mt.task_id] = OpSpec(mt.task_id, op, "fused", sample, reference, baseline,
                                           _seed_source(mt.task_id, p, n_aux), mt.shapes, mt.family, mt.dtype)


def mint(n: int = 4, seed: int = 0) -> List[str]:
    """Mint and register ``n`` tasks (deterministic for a seed)."""
    return TaskMinter(seed).mint(n)


def materialize(task_id: str, root: str) -> str:
    """Write a registered (e.g. minted) spec to ``root/<task_id>/`` in the task
    ABI (task.yaml, reference.py, seed kernel) and reload it as a self-check."""
    import inspect
    import os

    import yaml

    from ..tasks.base import Task
    from ..tasks.ops_library import SPECS
    spec = SPECS[task_id]
    d = os.path.join(root, task_id)
    os.makedirs(d, exist_ok=True)
    shapes = {k: spec.shapes[k] for k in ("minimal", "primary") if k in spec.shapes}
    shapes["validation"] = list(spec.shapes.get("validation", []) or [])
    y = {"task_id": task_id, "operation": spec.operation, "dtype": spec.dtype, "backend": "triton",
         "gpu_target": "sm_100a", "seed_kernel_name": "seed_kernel.py", "entry": spec.entry, "spec": task_id,
         "snr_threshold": spec.snr_threshold, "family": spec.family, "shapes": shapes,
         "targets": {"comparison_baseline": "torch eager in the task dtype"}}
    with open(os.path.join(d, "task.yaml"), "w") as f:
        yaml.safe_dump(y, f, sort_keys=False)
    with open(os.path.join(d, "seed_kernel.py"), "w") as f:
        f.write(spec.seed_src)
    try:
        ref = inspect.getsource(spec.reference)
    except (OSError, TypeError):
        ref = f"# reference: {task_id} (generated composition)\n"
    with open(os.path.join(d, "reference.py"), "w") as f:
        f.write(ref)
    t = Task.from_dir(d)
    if t.task_id != task_id or [s.dims for s in t.shapes][:1] != [shapes["minimal"]]:
        raise ValueError(f"materialize self-check failed for {task_id}")
    return d
