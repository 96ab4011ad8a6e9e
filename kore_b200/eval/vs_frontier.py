"""Head-to-head: our policy against a frontier model on the same tasks.

Both arms get the same attempt budget per task through the verified
environment. Per task the winner is decided by correctness first, then by
the worst-shape speedup over the vendor baseline, with a tie band
(``tie_margin``, 2% by default) so timing noise does not pick winners. The
report gives win / tie / loss counts, the win rate over decided tasks with a
Wilson 95% interval, an exact two-sided sign test, fast_p at 1.0 / 1.2 /
1.5x for both arms and the per-task table. A frontier endpoint that fails is
reported as ``unavailable`` (its tasks are left out of the comparison), never
scored as a loss for it.

    python -m kore_b200.eval.vs_frontier --model ckpt/ --frontier-url http://host/v1 --frontier-model NAME

Reference parity: kore/eval/vs_opus.py (winner_for_task, head_to_head
win rate, fast_p comparison, report) for any OpenAI-compatible frontier model.
"""
from __future__ import annotations

import argparse
import json
import math
from typing import Callable, Dict, List, Optional, Sequence

from .metrics import fast_p, sign_test
from .policies import FrontierUnavailable


def winner_for_task(ours: Optional[dict], theirs: Optional[dict], tie_margin: float = 1.02) -> str:
    """"ours" | "theirs" | "tie" | "unavailable" for one task's best results
    ({"correct", "speedup"}; None when that arm could not run)."""
    if ours is None or theirs is None:
        return "unavailable"
    oc, tc = bool(ours.get("correct")), bool(theirs.get("correct"))
    if oc != tc:
        return "ours" if oc else "theirs"
    if not oc:
        return "tie"
    a, b = float(ours.get("speedup") or 0.0), float(theirs.get("speedup") or 0.0)
    if a > b * tie_margin:
        return "ours"
    if b > a * tie_margin:
        return "theirs"
    return "tie"


def wilson(k: int, n: int, z: float = 1.96):
    if n == 0:
        return (float("nan"), float("nan"))
    p = k / n
    d = 1 + z * z / n
    c = (p + z * z / (2 * n)) / d
    h = z * math.sqrt(p * (1 - p) / n + z * z / (4 * n * n)) / d
    return (max(0.0, c - h), min(1.0, c + h))


def compare(ours: Sequence[dict], theirs: Sequence[Optional[dict]], tie_margin: float = 1.02) -> dict:
    """``ours[i]`` / ``theirs[i]`` are the two arms' best results on task i."""
    per = []
    for o, t in zip(ours, theirs):
        per.append({"task_id": (o or t or {}).get("task_id"), "winner": winner_for_task(o, t, tie_margin),
                    "ours": (o or {}).get("speedup"), "theirs": (t or {}).get("speedup") if t else None})
    w = sum(p["winner"] == "ours" for p in per)
    l = sum(p["winner"] == "theirs" for p in per)
    ties = sum(p["winner"] == "tie" for p in per)
    un = sum(p["winner"] == "unavailable" for p in per)
    both = [(o, t) for o, t in zip(ours, theirs) if o is not None and t is not None]
    a = [(o.get("speedup") or 0.0) if o.get("correct") else 0.0 for o, _ in both]
    b = [(t.get("speedup") or 0.0) if t.get("correct") else 0.0 for _, t in both]
    dec = w + l
    return {"wins": w, "losses": l, "ties": ties, "unavailable": un,
            "win_rate": (w / dec) if dec else float("nan"), "win_rate_ci95": wilson(w, dec),
            "sign_test_p": sign_test(a, b) if both else float("nan"),
            "fast_p": {f"{p}": {"ours": fast_p([o for o, _ in both], p), "theirs": fast_p([t for _, t in both], p)}
                       for p in (1.0, 1.2, 1.5)},
            "per_task": per}


def head_to_head(ours_policy: Callable, theirs_policy: Callable, tasks, env_factory, budget: int = 1,
                 tie_margin: float = 1.02) -> dict:
    from .bakeoff import evaluate_policy
    ours = evaluate_policy(ours_policy, tasks, env_factory, budget)
    theirs: List[Optional[dict]] = []
    for t in tasks:
        try:
            theirs += evaluate_policy(theirs_policy, [t], env_factory, budget)
        except FrontierUnavailable:
            theirs.append(None)
    return compare(ours, theirs, tie_margin)


def format_report(res: dict, names=("ours", "frontier")) -> str:
    lo, hi = res["win_rate_ci95"]
    lines = [f"# {names[0]} vs {names[1]}", "",
             f"wins {res['wins']}, losses {res['losses']}, ties {res['ties']}, unavailable {res['unavailable']}",
             f"win rate over decided tasks: {res['win_rate']:.2f} (95% CI {lo:.2f}-{hi:.2f}); "
             f"sign test p = {res['sign_test_p']:.3g}", "",
             f"| fast_p | {names[0]} | {names[1]} |", "|---|---|---|"]
    for p, v in res["fast_p"].items():
        lines.append(f"| {p}x | {v['ours']:.2f} | {v['theirs']:.2f} |")
    lines += ["", "| task | winner | speedup ours | speedup theirs |", "|---|---|---|---|"]
    for r in res["per_task"]:
        f = (lambda x: "-" if x is None else f"{x:.2f}")
        lines.append(f"| {r['task_id']} | {r['winner']} | {f(r['ours'])} | {f(r['theirs'])} |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore eval vs-frontier")
    ap.add_argument("--model", required=True)
    ap.add_argument("--frontier-url", required=True)
    ap.add_argument("--frontier-model", required=True)
    ap.add_argument("--tasks", default="", help="task ids (default: the held-out split)")
    ap.add_argument("--budget", type=int, default=1)
    ap.add_argument("--turns", type=int, default=1)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    from ..data.teacher import LocalTeacher
    from ..env.kore_env import KoreEnv
    from ..tasks.registry import get_task, split_tasks
    from .policies import frontier_policy, model_policy
    ids = [t for t in a.tasks.split(",") if t] or split_tasks()[1]
    tasks = [get_task(t) for t in ids]
    envf = lambda t: KoreEnv(t)                                          # noqa: E731
    ours = model_policy(LocalTeacher(a.model).generate, turns=a.turns, env_factory=envf)
    theirs = frontier_policy(url=a.frontier_url, model=a.frontier_model, turns=a.turns, env_factory=envf)
    res = head_to_head(ours, theirs, tasks, envf, a.budget)
    print(format_report(res, ("ours", a.frontier_model)))
    if a.out:
        with open(a.out, "w") as f:
            json.dump(res, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
