"""Task minter: composes new fused-operator tasks from a typed grammar of
verified torch primitives (elementwise unary/binary, row reductions,
normalisations, matmul), checks them with a construction gate (finite
outputs, shape preservation, non-trivial dependence on every input,
deterministic, roofline-modelable, bounded size) and registers them as
library specs with a naive Triton-free seed (the policy writes the kernel).
Reference parity: kore/openended/grammar.py:82-590, minter.py:323-399,
materialize.py:232."""
from __future__ import annotations

import random
from typing import Callable, List, Optional, Tuple

import torch

from ..tasks.ops_library import OpSpec, SPECS

UNARY = {"relu": torch.relu, "silu": torch.nn.functional.silu, "tanh": torch.tanh, "sigmoid": torch.sigmoid,
         "square": torch.square}
BINARY = {"add": torch.add, "mul": torch.mul, "sub": torch.sub, "max": torch.maximum}
ROW = {"softmax": lambda x: torch.softmax(x, -1),
       "rmsnorm": lambda x: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6),
       "logsumexp_center": lambda x: x - torch.logsumexp(x, -1, keepdim=True)}


def mint_expression(rng: random.Random, depth: int = 2) -> Tuple[str, Callable]:
    """Random composition f(a, b) of primitives; returns (name, fn)."""
    name, fn = "a", (lambda a, b: a)
    for _ in range(depth):
        kind = rng.choice(["u", "b", "r"])
        if kind == "u":
            n, f = rng.choice(list(UNARY.items()))
            name, fn = f"{n}({name})", (lambda g, f=f: (lambda a, b: f(g(a, b))))(fn)
        elif kind == "b":
            n, f = rng.choice(list(BINARY.items()))
            name, fn = f"{n}({name},b)", (lambda g, f=f: (lambda a, b: f(g(a, b), b)))(fn)
        else:
            n, f = rng.choice(list(ROW.items()))
            name, fn = f"{n}({name})", (lambda g, f=f: (lambda a, b: f(g(a, b))))(fn)
    return name, fn


def construction_gate(fn: Callable, dims=(64, 256)) -> Optional[str]:
    a = torch.randn(*dims)
    b = torch.randn(*dims)
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
    if y.abs().max() == 0:
        return "trivial output"
    return None


def mint(n: int = 4, seed: int = 0) -> List[str]:
    rng = random.Random(seed)
    made = []
    tries = 0
    while len(made) < n and tries < 50 * n:
        tries += 1
        name, fn = mint_expression(rng, rng.randint(2, 3))
        if construction_gate(fn):
            continue
        tid = "minted_" + "".join(ch if ch.isalnum() else "_" for ch in name)[:60]
        if tid in SPECS:
            continue

        def mk(d, s, dev, dt):
            g = torch.Generator(device=dev)
            g.manual_seed(s)
            sh = (d["M"], d["N"])
            return (torch.randn(sh, generator=g, device=dev).to(dt), torch.randn(sh, generator=g, device=dev).to(dt))

        ref = (lambda f: (lambda a, b: f(a.float(), b.float())))(fn)
        seed_src = ("import torch\n\n\ndef fused(a, b):\n    raise NotImplementedError('write the fused kernel for "
                    f"{name}')\n")
        SPECS[tid] = OpSpec(tid, "elementwise", "fused", mk, ref, (lambda f: (lambda a, b: f(a, b)))(fn), seed_src,
                            {"minimal": {"M": 64, "N": 256}, "primary": {"M": 4096, "N": 4096}, "validation": []},
                            "minted")
        made.append(tid)
    return made


def materialize(task_id: str, root: str) -> str:
    """Write a registered (e.g. minted) spec to ``root/<task_id>/`` in the task
    ABI (task.yaml, reference.py, seed kernel) and self-check that the
    directory loads back with the same shapes (reference parity:
    kore/openended/materialize.py:232)."""
    import inspect
    import os

    import yaml

    from ..tasks.base import Task
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
        ref = f"# reference: {task_id} (generated expression)\n"
    with open(os.path.join(d, "reference.py"), "w") as f:
        f.write(ref)
    t = Task.from_dir(d)
    assert t.task_id == task_id and [s.dims for s in t.shapes][:1] == [shapes["minimal"]], "materialize self-check"
    return d
