"""Evaluation suites on top of the verified environment.

* ``robust_eval``: re-verifies and re-times a candidate over several
  independent trials (fresh environment, shuffled shape order) and keeps the
  worst speedup, so a lucky timing window cannot make a kernel look fast.
* ``champion_reeval``: re-measures the best kernel per task from a wins file
  and keeps only those that still beat the baseline by ``min_speedup``.
* ``head_to_head``: two policies on the same tasks and budget; per-task
  winner, win rate, and paired statistics on the speedups.
* ``korebench``: a fixed, versioned task list (one per operator family of
  the library) scored by fast_p at 1.0 / 1.2 / 1.5 and geometric-mean speedup.
* ``write_report``: markdown summary of any of the above.
Reference parity: kore/eval/champion.py:240, robust_eval.py:512,
head_to_head.py / vs_opus.py, korebench.py:32, report.py.
"""
from __future__ import annotations

import math
import random
from typing import Callable, Dict, List, Optional, Sequence

from ..reward.reward import worst_speedup
from .metrics import bootstrap_ci, fast_p, sign_test, wilcoxon

KOREBENCH_V1 = ("rmsnorm_bf16", "layernorm_bf16", "softmax_bf16", "silu_mul_bf16", "gemm_bf16",
                "flash_attn_decode_bf16", "rope_bf16", "topk_softmax_fp32", "cross_entropy_bf16",
                "genb_norm_add_rmsnorm_bf16", "genb_gemm_silu_up14b_bf16", "genb_moe_combine_d2048k8_bf16",
                "genb_train_adamw_n16m_bf16", "genb_sample_topp_mask_v151936_fp32", "genb_reduce_logsumexp_bf16")


def robust_eval(task, src: str, env_factory, trials: int = 3, seed: int = 0) -> Dict:
    rng = random.Random(seed)
    speeds, correct = [], True
    for _ in range(trials):
        env = env_factory(task)
        if hasattr(env, "shuffle_shapes"):
            env.shuffle_shapes(rng)
        obs = env.step(src)
        correct = correct and bool(obs.validation_passed)
        su = worst_speedup(obs) if obs.validation_passed else None
        speeds.append(su or 0.0)
    return {"task_id": task.task_id, "correct": correct, "speedup": min(speeds) if correct else 0.0,
            "speedups": speeds}


def champion_reeval(wins, tasks_by_id: Dict, env_factory, min_speedup: float = 1.0, trials: int = 2) -> List[Dict]:
    best: Dict[str, object] = {}
    for w in wins:
        if w.final_kernel and (w.task_id not in best or (w.speedup or 0) > (best[w.task_id].speedup or 0)):
            best[w.task_id] = w
    out = []
    for tid, w in sorted(best.items()):
        if tid not in tasks_by_id:
            continue
        r = robust_eval(tasks_by_id[tid], w.final_kernel, env_factory, trials)
        r["claimed"] = w.speedup
        r["kept"] = r["correct"] and r["speedup"] >= min_speedup
        out.append(r)
    return out


def head_to_head(policy_a: Callable, policy_b: Callable, tasks, env_factory, budget: int = 1) -> Dict:
    from .bakeoff import evaluate_policy
    ra = evaluate_policy(policy_a, tasks, env_factory, budget)
    rb = evaluate_policy(policy_b, tasks, env_factory, budget)
    a = [r["speedup"] for r in ra]
    b = [r["speedup"] for r in rb]
    wins = sum(x > y for x, y in zip(a, b))
    ties = sum(x == y for x, y in zip(a, b))
    return {"a_win_rate": wins / max(1, len(a)), "ties": ties, "mean_diff_ci": bootstrap_ci(a, b),
            "sign_p": sign_test(a, b), "wilcoxon_p": wilcoxon(a, b), "per_task": list(zip([r["task_id"] for r in ra], a, b))}


def korebench(policy: Callable, env_factory, task_ids: Sequence[str] = KOREBENCH_V1, budget: int = 1) -> Dict:
    from ..tasks.registry import get_task
    from .bakeoff import evaluate_policy
    tasks = [get_task(t) for t in task_ids]
    res = evaluate_policy(policy, tasks, env_factory, budget)
    sp = [r["speedup"] for r in res if r["correct"] and r["speedup"] > 0]
    return {"version": "v1", "n": len(res), "fast_1.0": fast_p(res, 1.0), "fast_1.2": fast_p(res, 1.2),
            "fast_1.5": fast_p(res, 1.5), "geomean_speedup_correct": math.exp(sum(map(math.log, sp)) / len(sp)) if sp else 0.0,
            "results": res}


def write_report(path: str, title: str, sections: Dict[str, Dict]) -> str:
    lines = [f"# {title}", ""]
    for name, d in sections.items():
        lines += [f"## {name}", "", "| key | value |", "|---|---|"]
        for k, v in d.items():
            if isinstance(v, (list, dict)):
                continue
            lines.append(f"| {k} | {round(v, 4) if isinstance(v, float) else v} |")
        lines.append("")
    text = "\n".join(lines)
    with open(path, "w") as f:
        f.write(text)
    return text


def champion_verdict(claimed: Optional[float], *, correct: bool, correct_unseen: bool = True,
                     hack_reason: Optional[str] = None, cv_pct: Optional[float] = None,
                     speedup: Optional[float] = None, collapse: float = 0.7, max_cv_pct: float = 5.0) -> Dict:
    """Certify a champion kernel re-measured under harder conditions than
    training: correct on the training shapes AND on unseen shapes, no static
    reward hack, low timing variance, and a re-measured speedup that did not
    collapse below ``collapse`` x the claimed one."""
    reasons = []
    if not correct:
        reasons.append("incorrect on the training shapes")
    if not correct_unseen:
        reasons.append("incorrect on unseen shapes")
    if hack_reason:
        reasons.append(f"static check: {hack_reason}")
    if cv_pct is not None and cv_pct > max_cv_pct:
        reasons.append(f"timing variance {cv_pct:.1f}% > {max_cv_pct}%")
    if claimed and (speedup or 0.0) < collapse * claimed:
        reasons.append(f"speedup {speedup or 0.0:.2f}x collapsed below {collapse} x claimed {claimed:.2f}x")
    return {"certified": not reasons, "reasons": reasons, "claimed": claimed, "remeasured": speedup}
