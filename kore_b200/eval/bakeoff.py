"""Matched-budget bake-off: each policy gets the same number of verified
attempts per task; reports fast_p at 1.0/1.2/1.5x, mean worst-shape
speedup, and paired statistics between two arms. Generalisation split:
asserts no held-out task leaks into training data. Reference parity:
kore/eval/bakeoff.py:296, generalization.py:149-186."""
from __future__ import annotations

from typing import Callable, Dict, List, Sequence

from ..reward.reward import worst_speedup
from .metrics import bootstrap_ci, fast_p, sign_test, wilcoxon


def evaluate_policy(policy: Callable[[object], List[str]], tasks, env_factory, budget: int = 4) -> List[Dict]:
    out = []
    for t in tasks:
        env = env_factory(t)
        best = {"task_id": t.task_id, "correct": False, "speedup": 0.0}
        for src in policy(t)[:budget]:
            obs = env.step(src)
            if obs.validation_passed:
                su = worst_speedup(obs) or 0.0
                if su > best["speedup"]:
                    best = {"task_id": t.task_id, "correct": True, "speedup": su}
        out.append(best)
    return out


def matched_budget_bakeoff(arms: Dict[str, Callable], tasks, env_factory, budget: int = 4) -> Dict:
    res = {n: evaluate_policy(p, tasks, env_factory, budget) for n, p in arms.items()}
    summary = {n: {f"fast_{p}": fast_p(r, p) for p in (1.0, 1.2, 1.5)} for n, r in res.items()}
    names = list(res)
    if len(names) == 2:
        a = [r["speedup"] for r in res[names[0]]]
        b = [r["speedup"] for r in res[names[1]]]
        summary["paired"] = {"mean_diff_ci": bootstrap_ci(a, b), "sign_p": sign_test(a, b), "wilcoxon_p": wilcoxon(a, b)}
    return {"results": res, "summary": summary}


def assert_no_leakage(train_task_ids: Sequence[str], heldout_ids: Sequence[str]) -> None:
    leak = set(train_task_ids) & set(heldout_ids)
    if leak:
        raise AssertionError(f"held-out tasks leaked into training: {sorted(leak)[:5]}")
