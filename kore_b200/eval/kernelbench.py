"""KernelBench adapter and the held-out protocol.

KernelBench problems are PyTorch modules (``class Model(nn.Module)`` with a
``forward``, plus ``get_inputs()`` / ``get_init_inputs()``): the eager module
is both the correctness oracle and the baseline, and results are reported as
``fast_p`` (correct and more than p times faster than eager) at p = 1.0, 1.5
and 2.0. This module

* turns a problem into a task of this package (:func:`spec_to_task`): the
  module's forward in fp32 is the oracle, the eager forward in the task dtype
  is the baseline, and the problem source is the seed, so a KernelBench run
  goes through the same verified, L2-flushed timing pipeline as every task;
* loads real KernelBench problem files from a checkout
  (:func:`load_kernelbench_dir`, level directories of ``<n>_<name>.py``) and
  ships a handful of small bundled problems for offline tests;
* reports a policy's results in KernelBench's format
  (:func:`kernelbench_report`), per level;
* proposes a held-out split stratified over operator family, shape regime and
  dtype (:func:`propose_heldout`) and asserts that no held-out task, nor any
  task of a held-out family, is in the training set (:func:`assert_no_leakage`).

Reference behaviour: kore/eval/kernelbench_amd.py:68-707 and
kore/eval/generalization.py:107-186, with the sm_100a target.
"""
from __future__ import annotations

import importlib.util
import math
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence

import torch

KERNELBENCH_PS = (1.0, 1.5, 2.0)
TARGET = "sm_100a"


@dataclass
class KernelBenchSpec:
    name: str
    level: int
    source: str                    # the problem file (defines Model, get_inputs, get_init_inputs)
    dtype: str = "fp32"
    operation: str = "kernelbench"


_BUNDLED = {
    ("relu", 1): '''import torch
import torch.nn as nn


class Model(nn.Module):
    def forward(self, x):
        return torch.relu(x)


def get_inputs():
    return [torch.randn(4096, 4096)]


def get_init_inputs():
    return []
''',
    ("matmul", 1): '''import torch
import torch.nn as nn


class Model(nn.Module):
    def forward(self, a, b):
        return a @ b


def get_inputs():
    return [torch.randn(1024, 2048), torch.randn(2048, 1024)]


def get_init_inputs():
    return []
''',
    ("gemm_bias_gelu", 2): '''import torch
import torch.nn as nn


class Model(nn.Module):
    def __init__(self, n_in, n_out):
        super().__init__()
        self.lin = nn.Linear(n_in, n_out)

    def forward(self, x):
        return torch.nn.functional.gelu(self.lin(x))


def get_inputs():
    return [torch.randn(2048, 1024)]


def get_init_inputs():
    return [1024, 4096]
''',
    ("rmsnorm_residual", 2): '''import torch
import torch.nn as nn


class Model(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.w = nn.Parameter(torch.ones(d))

    def forward(self, x, r):
        h = x + r
        return h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * self.w


def get_inputs():
    return [torch.randn(4096, 2048), torch.randn(4096, 2048)]


def get_init_inputs():
    return [2048]
''',
    ("softmax", 1): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def forward(self, x):
        return torch.softmax(x, dim=-1)


def get_inputs():
    return [torch.randn(4096, 8192)]


def get_init_inputs():
    return []
''',
    ("layernorm", 1): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        return self.ln(x)


def get_inputs():
    return [torch.randn(8192, 1024)]


def get_init_inputs():
    return [1024]
''',
    ("sum_reduce", 1): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def forward(self, x):
        return x.sum(dim=1)


def get_inputs():
    return [torch.randn(2048, 16384)]


def get_init_inputs():
    return []
''',
    ("conv2d", 1): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, cin, cout, k):
        super().__init__()
        self.conv = nn.Conv2d(cin, cout, k, padding=k // 2)

    def forward(self, x):
        return self.conv(x)


def get_inputs():
    return [torch.randn(16, 64, 56, 56)]


def get_init_inputs():
    return [64, 128, 3]
''',
    ("batched_matmul", 1): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def forward(self, a, b):
        return torch.bmm(a, b)


def get_inputs():
    return [torch.randn(32, 512, 256), torch.randn(32, 256, 512)]


def get_init_inputs():
    return []
''',
    ("swiglu_mlp", 2): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.gate = nn.Linear(d, f, bias=False)
        self.up = nn.Linear(d, f, bias=False)
        self.down = nn.Linear(f, d, bias=False)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


def get_inputs():
    return [torch.randn(1024, 1024)]


def get_init_inputs():
    return [1024, 2816]
''',
    ("matmul_scale_residual", 2): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, n_in, n_out, scale):
        super().__init__()
        self.lin = nn.Linear(n_in, n_out)
        self.scale = scale

    def forward(self, x, r):
        return self.lin(x) * self.scale + r


def get_inputs():
    return [torch.randn(2048, 1024), torch.randn(2048, 1024)]


def get_init_inputs():
    return [1024, 1024, 0.5]
''',
    ("conv_bn_relu", 2): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.conv = nn.Conv2d(c, c, 3, padding=1, bias=False)
        self.bn = nn.BatchNorm2d(c)

    def forward(self, x):
        return torch.relu(self.bn(self.conv(x)))


def get_inputs():
    return [torch.randn(8, 64, 64, 64)]


def get_init_inputs():
    return [64]
''',
    ("attention_block", 3): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.h = h
        self.qkv = nn.Linear(d, 3 * d, bias=False)
        self.o = nn.Linear(d, d, bias=False)

    def forward(self, x):
        B, S, D = x.shape
        q, k, v = self.qkv(x).view(B, S, 3, self.h, D // self.h).permute(2, 0, 3, 1, 4)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.o(y.transpose(1, 2).reshape(B, S, D))


def get_inputs():
    return [torch.randn(2, 512, 512)]


def get_init_inputs():
    return [512, 8]
''',
    ("transformer_mlp_block", 3): '''import torch
import torch.nn as nn
import torch.nn.functional as F


class Model(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.ln = nn.LayerNorm(d)
        self.fc1 = nn.Linear(d, 4 * d)
        self.fc2 = nn.Linear(4 * d, d)

    def forward(self, x):
        return x + self.fc2(F.gelu(self.fc1(self.ln(x))))


def get_inputs():
    return [torch.randn(4, 256, 512)]


def get_init_inputs():
    return [512]
''',
}


def bundled_specs() -> List[KernelBenchSpec]:
    return [KernelBenchSpec(f"kb_l{lvl}_{n}", lvl, src) for (n, lvl), src in _BUNDLED.items()]


def _load_module(spec: KernelBenchSpec):
    ns: dict = {}
    exec(compile(spec.source, spec.name, "exec"), ns)
    return ns


def spec_to_task(spec: KernelBenchSpec, dtype: str = "bf16"):
    """A task of this package whose oracle/baseline are the problem's module."""
    from ..tasks.base import Shape, Task
    from ..tasks.ops_library import SPECS
    from ..tasks.spec import OpSpec
    ns = _load_module(spec)
    torch.manual_seed(0)
    init = ns["get_init_inputs"]()
    model = ns["Model"](*init)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]

    def mk(d, seed, dev, t):
        torch.manual_seed(seed)
        return tuple(x.to(dev).to(t) if x.is_floating_point() else x.to(dev) for x in ns["get_inputs"]())

    def reference(*x):
        m = model.to(x[0].device).float()
        with torch.no_grad():
            return m(*(t.float() if t.is_floating_point() else t for t in x)).float()

    def baseline(*x):
        m = model.to(x[0].device).to(dt)
        with torch.no_grad():
            return m(*x)

    seed = spec.source + ("\n\ndef kernel(*inputs):\n    torch.manual_seed(0)\n"
                          "    m = Model(*get_init_inputs()).to(inputs[0].device).to(inputs[0].dtype)\n"
                          "    with torch.no_grad():\n        return m(*inputs)\n")
    tid = f"{spec.name}_{dtype}"
    SPECS[tid] = OpSpec(tid, spec.operation, "kernel", mk, reference, baseline, seed,
                        {"minimal": {"P": 0}, "primary": {"P": 0}}, f"kernelbench_l{spec.level}", dtype, 25.0)
    return Task(task_id=tid, operation=spec.operation, dtype=dtype, entry="kernel", spec=tid, snr_threshold=25.0,
                shapes=[Shape("primary", {"P": 0})], seed_src=seed, reference_src=spec.source,
                family=f"kernelbench_l{spec.level}",
                targets={"comparison_baseline": "torch_eager", "gpu_target": TARGET})


def load_kernelbench_dir(root: str, levels: Sequence[int] = (1, 2)) -> List[KernelBenchSpec]:
    """Problems from a KernelBench checkout: ``<root>/level<k>/<n>_<name>.py``."""
    out = []
    for lvl in levels:
        d = Path(root) / f"level{lvl}"
        for p in sorted(d.glob("*.py")) if d.is_dir() else []:
            src = p.read_text()
            if "class Model" in src and "def get_inputs" in src:
                out.append(KernelBenchSpec(f"kb_l{lvl}_{p.stem}", lvl, src))
    return out


def _fastp(results: Sequence[dict], p: float) -> float:
    if not results:
        return 0.0
    return sum(1 for r in results if r.get("correct") and (r.get("speedup") or 0.0) > p) / len(results)


def kernelbench_report(results: Sequence[dict], specs: Optional[Sequence[KernelBenchSpec]] = None) -> Dict:
    """fast_p at p in {1.0, 1.5, 2.0}, overall and per level."""
    rep = {"target": TARGET, "baseline": "torch_eager", "n": len(results),
           **{f"fast_{p}": _fastp(results, p) for p in KERNELBENCH_PS}}
    if specs:
        lv = {s.name: s.level for s in specs}
        by: Dict[int, List[dict]] = {}
        for r in results:
            name = str(r.get("task_id", "")).rsplit("_", 1)[0]
            by.setdefault(lv.get(name, 0), []).append(r)
        rep["levels"] = {f"level{k}": {f"fast_{p}": _fastp(v, p) for p in KERNELBENCH_PS} | {"n": len(v)}
                         for k, v in sorted(by.items())}
    sp = [r["speedup"] for r in results if r.get("correct") and (r.get("speedup") or 0) > 0]
    rep["geomean_speedup_correct"] = math.exp(sum(map(math.log, sp)) / len(sp)) if sp else 0.0
    return rep


def run_kernelbench(policy: Callable, specs: Sequence[KernelBenchSpec], env_factory, dtype: str = "bf16",
                    budget: int = 1) -> Dict:
    from .bakeoff import evaluate_policy
    tasks = [spec_to_task(s, dtype) for s in specs]
    res = evaluate_policy(policy, tasks, env_factory, budget)
    return kernelbench_report(res, specs)


# ----------------------------------------------------------------------------- held-out protocol
def shape_regime(task) -> str:
    sizes = [math.prod(v for v in s.dims.values() if isinstance(v, int) and v > 0) for s in task.shapes]
    odd = any(any(isinstance(v, int) and v % 8 for v in s.dims.values()) for s in task.shapes)
    big = max(sizes or [0])
    return ("odd" if odd else "aligned") + ("_large" if big >= (1 << 24) else "_small")


@dataclass
class HeldoutProtocol:
    heldout_families: List[str]
    heldout_tasks: List[str]
    train_tasks: List[str]
    strata: Dict[str, int] = field(default_factory=dict)


def propose_heldout(tasks: Optional[Sequence] = None, *, families: Sequence[str] = ("attention", "ssm"),
                    frac: float = 0.08, seed: int = 0) -> HeldoutProtocol:
    """Whole families held out, plus a stratified sample over (family, shape
    regime, dtype) of the rest."""
    if tasks is None:
        from ..tasks.registry import all_tasks
        tasks = all_tasks()
    rng = random.Random(seed)
    fam_out = set(families)
    held, strata = [], {}
    groups: Dict[tuple, List[str]] = {}
    for t in tasks:
        if t.family in fam_out:
            held.append(t.task_id)
            continue
        groups.setdefault((t.family, shape_regime(t), t.dtype), []).append(t.task_id)
    for key, ids in sorted(groups.items()):
        k = int(round(frac * len(ids)))
        pick = rng.sample(sorted(ids), k) if k else []
        held += pick
        if pick:
            strata["/".join(key)] = len(pick)
    held_set = set(held)
    train = sorted(t.task_id for t in tasks if t.task_id not in held_set)
    return HeldoutProtocol(sorted(fam_out), sorted(held_set), train, strata)


def leakage(protocol: HeldoutProtocol, tasks: Optional[Sequence] = None) -> Dict[str, List[str]]:
    if tasks is None:
        from ..tasks.registry import all_tasks
        tasks = all_tasks()
    fam = {t.task_id: t.family for t in tasks}
    train = set(protocol.train_tasks)
    return {"heldout_in_train": sorted(train & set(protocol.heldout_tasks)),
            "heldout_family_in_train": sorted(t for t in train if fam.get(t) in set(protocol.heldout_families))}


def assert_no_leakage(protocol: HeldoutProtocol, tasks: Optional[Sequence] = None) -> None:
    bad = leakage(protocol, tasks)
    if any(bad.values()):
        raise AssertionError(f"held-out leakage: {bad}")
