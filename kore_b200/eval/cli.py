"""``kore eval`` — evaluate a policy checkpoint on the held-out kernel tasks
(fast_p, worst-shape speedups) with the verified environment."""
from __future__ import annotations

import argparse
import json


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore eval")
    ap.add_argument("--model", required=True, help="checkpoint dir or 'seed' (the seed kernels)")
    ap.add_argument("--split", default="heldout", choices=["heldout", "train", "all"])
    ap.add_argument("--budget", type=int, default=1)
    ap.add_argument("--turns", type=int, default=1, help="model turns per attempt, with verifier feedback between")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    from ..env.kore_env import KoreEnv
    from ..tasks.registry import all_tasks, get_task, split_tasks
    from .bakeoff import evaluate_policy
    from .metrics import fast_p
    tr, ho = split_tasks()
    ids = {"heldout": ho, "train": tr, "all": tr + ho}[a.split]
    tasks = [get_task(t) for t in ids]
    from .policies import model_policy, seed_policy
    if a.model == "seed":
        policy = seed_policy
    else:
        from ..data.teacher import LocalTeacher
        one = model_policy(LocalTeacher(a.model).generate, turns=a.turns, env_factory=lambda t: KoreEnv(t))

        def policy(t):
            return [src for _ in range(a.budget) for src in one(t)]
    res = evaluate_policy(policy, tasks, lambda t: KoreEnv(t), a.budget * max(1, a.turns))
    out = {"fast_1.0": fast_p(res, 1.0), "fast_1.2": fast_p(res, 1.2), "results": res}
    print(json.dumps(out))
    if a.out:
        json.dump(out, open(a.out, "w"), indent=2)
    return 0
