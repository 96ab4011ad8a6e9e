"""Zero-shot transfer to held-out operator families.

``classify(task)`` puts a task in one of eight families by first-matching
rules on its id and operation (attention, moe, gemm, norm, positional, quant,
reduction, activation; ``other`` when none matches). ``family_split`` holds
out whole families (never a partial one) and checks that no held-out task is
in the training list. ``leave_one_family_out`` fits any scoring model on all
families but one and reports its fit on the held-out family (e.g. the physics
residual reward against measured speedups), so transfer is measured the same
way for every family. ``heldout_report`` aggregates a policy's results by
family, counting only kernels the reward itself judged correct.

This is the analysis taxonomy; the product train / held-out split is the task
registry's (``kore_b200.tasks.registry.split_tasks``).
Reference behaviour: kore/eval/generalization.py:107-186.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

FAMILY_RULES: Tuple[Tuple[str, Tuple[str, ...]], ...] = (
    ("attention", ("attn", "attention", "mla", "paged", "decode", "prefill", "retention", "linear_attention")),
    ("moe", ("moe", "expert", "router", "topk_softmax", "grouped")),
    ("gemm", ("gemm", "matmul", "bmm", "linear", "conv", "newton_schulz")),
    ("norm", ("norm", "layernorm", "rmsnorm")),
    ("positional", ("rope", "rotary", "alibi", "position")),
    ("quant", ("quant", "fp8", "int8", "int4", "mxfp4", "nf4")),
    ("reduction", ("reduce", "sum", "softmax", "logsumexp", "entropy", "loss", "cumsum", "scan", "sort", "topk",
                   "argmax", "mean", "var", "std")),
    ("activation", ("relu", "gelu", "silu", "swish", "tanh", "sigmoid", "elementwise", "unary", "binary",
                    "activation", "mish", "softplus")),
)
FAMILIES = tuple(f for f, _ in FAMILY_RULES)


def classify(task) -> str:
    text = f"{getattr(task, 'task_id', task)} {getattr(task, 'operation', '')}".lower()
    for fam, keys in FAMILY_RULES:
        if any(k in text for k in keys):
            return fam
    return "other"


def family_split(tasks: Sequence, heldout: Sequence[str]) -> Tuple[List[str], List[str]]:
    ho = set(heldout)
    unknown = ho - set(FAMILIES) - {"other"}
    if unknown:
        raise ValueError(f"unknown families {sorted(unknown)}")
    train = [t.task_id for t in tasks if classify(t) not in ho]
    held = [t.task_id for t in tasks if classify(t) in ho]
    if set(train) & set(held):
        raise AssertionError("a task is on both sides of the split")
    return train, held


def _r2(y: Sequence[float], yhat: Sequence[float]) -> float:
    n = len(y)
    if n < 2:
        return float("nan")
    m = sum(y) / n
    ss_tot = sum((a - m) ** 2 for a in y)
    ss_res = sum((a - b) ** 2 for a, b in zip(y, yhat))
    return 1.0 - ss_res / ss_tot if ss_tot > 0 else float("nan")


def leave_one_family_out(rows: Sequence[Dict], fit: Callable[[Sequence[Dict]], Callable[[Dict], float]],
                         target: str = "y") -> Dict[str, Dict[str, float]]:
    """``rows``: {family, <features...>, y}; ``fit(train_rows) -> predict(row)``.
    Returns per held-out family its R^2 and the number of rows."""
    fams = sorted({r["family"] for r in rows})
    out = {}
    for f in fams:
        train = [r for r in rows if r["family"] != f]
        test = [r for r in rows if r["family"] == f]
        if not train or len(test) < 2:
            continue
        pred = fit(train)
        out[f] = {"r2": _r2([r[target] for r in test], [pred(r) for r in test]), "n": len(test)}
    vals = sorted(v["r2"] for v in out.values() if not math.isnan(v["r2"]))
    if vals:
        out["_median"] = {"r2": vals[len(vals) // 2], "n": sum(v["n"] for v in out.values())}
    return out


def heldout_report(results: Iterable[Dict], tasks_by_id: Dict[str, object], heldout: Sequence[str]) -> Dict:
    """fast_1 and mean gated speedup per family, correct kernels only (the
    reward's verdict), for held-out and training families separately."""
    from .fastp import gated_speedup
    by: Dict[str, List[Dict]] = {}
    for r in results:
        t = tasks_by_id.get(r.get("task_id"))
        if t is None:
            continue
        by.setdefault(classify(t), []).append(r)
    rep = {}
    for fam, rs in sorted(by.items()):
        ok = [gated_speedup(r.get("speedup"), r.get("cv_pct")) for r in rs if r.get("correct")]
        rep[fam] = {"n": len(rs), "heldout": fam in set(heldout),
                    "fast_1.0": sum(1 for s in ok if s > 1.0) / len(rs),
                    "mean_speedup_correct": sum(ok) / len(ok) if ok else 0.0}
    return rep
