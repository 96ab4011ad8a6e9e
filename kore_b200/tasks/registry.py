"""Task registry and the deterministic train / held-out split.

Tasks come from the operator library plus any ``*/task.yaml`` directories
under ``KORE_TASKS_DIR``. Whole families are held out (attention prefill and
the fp8 quantisation family) together with a seeded fraction of the rest,
so evaluation measures generalisation to unseen operators (reference:
kore/tasks/registry.py:39-213)."""
from __future__ import annotations

import glob
import os
import random
from typing import List, Optional, Tuple

from .base import Task
from .ops_library import SPECS

HELDOUT_FAMILIES = {"quant", "ssm", "sort_sparse"}
HELDOUT_TASKS = {"flash_attn_prefill_bf16", "gen_max_bf16"}
# held-out operator variants: every dtype / shape of these never appears in training
HELDOUT_PATTERNS = ("_sliding", "_softcap", "genb_unary_mish_", "genb_binary_hypot_", "genb_reduce_entropy_",
                    "genb_norm_rmsnorm_gated_", "genb_gemm_relu2_", "genb_train_lion_", "genb_sample_minp_")


def _discover_dirs() -> List[Task]:
    root = os.environ.get("KORE_TASKS_DIR")
    if not root:
        return []
    return [Task.from_dir(os.path.dirname(p)) for p in sorted(glob.glob(os.path.join(root, "*", "task.yaml")))]


def all_tasks() -> List[Task]:
    tasks = [Task.from_spec(s) for s in SPECS.values()]
    seen = {t.task_id for t in tasks}
    tasks += [t for t in _discover_dirs() if t.task_id not in seen]
    return tasks


def get_task(task_id: str) -> Task:
    for t in all_tasks():
        if t.task_id == task_id:
            return t
    raise KeyError(f"unknown task {task_id!r}")


def split_tasks(seed: int = 0, heldout_frac: float = 0.0) -> Tuple[List[str], List[str]]:
    ids = sorted(t.task_id for t in all_tasks())
    fam = {t.task_id: t.family for t in all_tasks()}
    held = {i for i in ids if fam[i] in HELDOUT_FAMILIES or i in HELDOUT_TASKS
            or any(p in i for p in HELDOUT_PATTERNS)}
    rest = [i for i in ids if i not in held]
    rng = random.Random(seed)
    extra = set(rng.sample(rest, int(round(heldout_frac * len(rest))))) if heldout_frac > 0 else set()
    held |= extra
    return [i for i in ids if i not in held], sorted(held)
