"""Smokes and proofs: small end-to-end checks a user runs before a campaign.

    python -m kore_b200.proofs <name> [--device cuda:0] [--limit N]

* ``env``        the verified environment grades a task's seed on the GPU
                 (compiles, correct on every shape, timed against the vendor);
* ``sft``        three SFT steps of a tiny model; the loss must fall;
* ``grpo``       one GRPO step of a tiny model on the synthetic reward env
                 (rollout, reference log-probs, update);
* ``breadth``    every breadth task's seed against its fp32 oracle on the
                 minimal shape (CPU is enough);
* ``ops``        every registered task has a roofline model and a seed that
                 executes;
* ``grpo-repro`` the ragged multi-process GRPO advantage step: gloo ranks
                 holding different numbers of trajectories per group agree
                 with the single-process computation.

Each prints one JSON line and exits 0 on success.
Reference behaviour: scripts/smoke_env.py, grpo_smoke.py, sft_smoke.py,
_repro_grpo_step.py, prove_new_ops.py, verify_breadth.py.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from typing import Dict, List, Optional

import torch


def smoke_env(task_id: str = "rmsnorm_bf16", device: str = "cuda:0") -> Dict[str, object]:
    if not torch.cuda.is_available():
        return {"ok": True, "skipped": "no GPU"}
    from .env.kore_env import KoreEnv
    from .tasks.registry import get_task
    t = get_task(task_id)
    obs = KoreEnv(t).step(t.seed_src)
    return {"ok": bool(obs.compiled and obs.validation_passed), "task": task_id, "wall_ms": obs.wall_ms,
            "baseline_ms": obs.baseline_ms, "snr_db": obs.snr_db}


def smoke_sft(device: str = "cpu", steps: int = 3) -> Dict[str, object]:
    from .engine.smoke import smoke_config
    from .engine.trainer import CausalLMTrainer
    from .parallel.dist import DistContext
    dev = torch.device(device)
    ctx = DistContext(device=dev)
    tr = CausalLMTrainer(smoke_config(), ctx, lr=3e-3, max_grad_norm=1.0, seed=0,
                         dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 2048, (2, 128), generator=g).to(dev)
    losses = [float(tr.train_step_device(ids)) for _ in range(steps)]
    return {"ok": losses[-1] < losses[0], "losses": [round(x, 4) for x in losses]}


def smoke_grpo(device: str = "cpu") -> Dict[str, object]:
    from .engine.smoke import smoke_config
    from .env.base import SyntheticRewardEnv
    from .models import Qwen3Weights
    from .parallel.dist import DistContext
    from .policy.configs import GRPOConfig
    from .policy.grpo import GRPOTrainer
    dev = torch.device(device)
    cfg = smoke_config()
    w = Qwen3Weights(cfg, device=dev, dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32, seed=0)
    gc = GRPOConfig(num_trajectories=4, num_turns=2, tasks_per_step=2, max_response_length=16,
                    max_prompt_length=512, learning_rate=1e-4, temperature=1.0, dynamic_sampling=False,
                    starpo_s=False, total_steps=1, overlong_mask=False, bf16=dev.type == "cuda")
    env = SyntheticRewardEnv(seed=0, prompt_len=48, feedback_len=8, vocab_size=cfg.vocab_size)
    tr = GRPOTrainer(gc, weights=w, env=env, ctx=DistContext(device=dev),
                     rollout_kwargs=dict(num_pages=64, page_size=64, max_seq_len=512))
    t0 = time.time()
    st = tr.train_step(["a", "b"])
    return {"ok": st["gen_tokens"] > 0 and st["samples"] > 0 and bool(torch.isfinite(torch.tensor(st["loss"]))),
            "samples": st["samples"], "gen_tokens": st["gen_tokens"], "loss": st["loss"],
            "seconds": round(time.time() - t0, 2)}


def verify_breadth(limit: Optional[int] = None, device: str = "cpu") -> Dict[str, object]:
    from .tasks.ops_library import SPECS
    names = sorted(n for n in SPECS if n.startswith("genb_"))[: limit or None]
    bad: List[str] = []
    for n in names:
        s = SPECS[n]
        try:
            x = s.make_inputs(s.shapes["minimal"], 0, device, torch.float32)
            ref = s.reference(*x)
            ns: dict = {}
            exec(s.seed_src, ns)
            out = ns[s.entry](*x)
            r = ref.float().nan_to_num(0, 0, 0)
            if tuple(out.shape) != tuple(ref.shape) or \
                    (out.float().nan_to_num(0, 0, 0) - r).abs().max() > 1e-2 * max(1.0, float(r.abs().max())):
                bad.append(n)
        except Exception as e:  # noqa: BLE001
            bad.append(f"{n}: {type(e).__name__}")
    return {"ok": not bad, "checked": len(names), "failed": bad[:20], "n_failed": len(bad)}


def prove_ops(limit: Optional[int] = None) -> Dict[str, object]:
    from .analysis.rooflines import flops_bytes
    from .tasks.registry import all_tasks
    # external KernelBench problems registered at run time carry no operation
    # model (their work is whatever the problem module does): no roofline to check
    ts = [t for t in all_tasks() if t.operation != "kernelbench"][: limit or None]
    no_roof, no_seed = [], []
    for t in ts:
        sh = t.shape("primary") or (t.shapes[0] if t.shapes else None)
        if sh is None or flops_bytes(t.operation, sh.dims, t.dtype) is None:
            no_roof.append(t.task_id)
        try:
            compile(t.seed_src, t.task_id, "exec")
        except SyntaxError:
            no_seed.append(t.task_id)
    return {"ok": not no_roof and not no_seed, "tasks": len(ts), "no_roofline": no_roof[:10],
            "seed_syntax_errors": no_seed[:10]}


def _repro_worker(rank: int, world: int, port: int, groups, q) -> None:
    import torch.distributed as dist

    from .parallel.dist import DistContext
    from .policy import rl_math as M
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctx = DistContext(rank=rank, world=world, backend="gloo")
    mine = [[r for i, r in enumerate(g) if i % world == rank] for g in groups]        # ragged shares
    gathered = [ctx.all_gather_object(m) for m in mine]
    adv = [M.distributed_group_advantages(g)[rank] for g in gathered]
    q.put((rank, adv))
    dist.barrier()
    dist.destroy_process_group()


def repro_grpo_step(world: int = 2, port: int = 29631) -> Dict[str, object]:
    import torch.multiprocessing as mp

    from .policy import rl_math as M
    groups = [[0.0, 1.0, 0.3, 0.3, 0.9], [1.0, 1.0, 0.1], [0.2, 0.4, 0.6, 0.8, 1.0, 0.0, 0.5]]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_repro_worker, args=(r, world, port, groups, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    ok = True
    for gi, g in enumerate(groups):
        shares = [[r for i, r in enumerate(g) if i % world == k] for k in range(world)]
        want = M.distributed_group_advantages(shares)
        for k in range(world):
            ok = ok and all(abs(a - b) < 1e-9 for a, b in zip(got[k][gi], want[k]))
    return {"ok": ok, "world": world, "groups": len(groups)}


def prove_value_cold_start(groups: int = 200, holdout: int = 50) -> Dict[str, object]:
    """The value model fitted on synthetic ranked groups orders fresh held-out
    groups like their ground truth (within-group Spearman above 0.3)."""
    from .value.features import synthesize_groups
    from .value.model import ValueModel
    from .value.rerank import groupwise_spearman
    m = ValueModel().fit_groups(synthesize_groups(groups, seed=0))

    def score(rows):
        return list(m.predict(m.featurize([r["source"] for r in rows], rows[0]["meta"]))["utility"])
    rho = groupwise_spearman(score, synthesize_groups(holdout, seed=99))
    return {"ok": rho > 0.3, "holdout_spearman": rho}


def prove_corpus(limit: int = 400) -> Dict[str, object]:
    """The task-corpus audit and every generated task's roofline, plus a small
    mid-training corpus from this repository's own sources."""
    from .data.midtrain_corpus import build_midtrain_corpus
    from .tasks.audit import audit
    r = audit()
    c = build_midtrain_corpus(None, sources=["tasks", "repo_kernels", "docs"], max_docs=limit)
    return {"ok": r.with_roofline == r.tasks - r.external and c["docs"] > 0, "tasks": r.tasks, "heldout": r.heldout,
            "corpus_docs": c["docs"], "corpus_by_source": c["by_source"]}


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="kore-proofs")
    ap.add_argument("name", choices=["env", "sft", "grpo", "breadth", "ops", "grpo-repro", "value", "corpus"])
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--task", default="rmsnorm_bf16")
    a = ap.parse_args(argv)
    fn = {"env": lambda: smoke_env(a.task, a.device), "sft": lambda: smoke_sft(a.device),
          "grpo": lambda: smoke_grpo(a.device), "breadth": lambda: verify_breadth(a.limit),
          "ops": lambda: prove_ops(a.limit), "grpo-repro": lambda: repro_grpo_step(),
          "value": lambda: prove_value_cold_start(), "corpus": lambda: prove_corpus()}[a.name]
    res = fn()
    print(json.dumps({"proof": a.name, **res}, default=str), flush=True)
    return 0 if res.get("ok") else 1


if __name__ == "__main__":
    sys.exit(main())
