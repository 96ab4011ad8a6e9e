"""Shared epoch / step / checkpoint loop of the supervised trainers.

Examples are split over ranks with a strided slice (identical global order
on every rank), grouped into optimizer steps of
``per_device_train_batch_size * gradient_accumulation_steps`` examples per
rank, and fed to a step function. Checkpoints ``checkpoint-<step>`` hold the
HF weights, ``trainer_state.json`` and each rank's optimizer shard, so a run
resumes mid-stage (reference: HF Trainer resume via latest_checkpoint,
kore/policy/configs.py:654-679).
"""
from __future__ import annotations

import math
import os
import random
from typing import Callable, List, Optional, Sequence

import torch

from ..models.hf_io import save_pretrained
from ..obs import get_logger
from .configs import latest_checkpoint

log = get_logger("policy.loop")


def plan_steps(n_examples: int, world: int, per_device: int, accum: int, epochs: float,
               max_steps: int = -1) -> int:
    per_step = max(1, per_device * accum * world)
    steps = int(math.ceil(n_examples * epochs / per_step))
    return min(steps, max_steps) if max_steps and max_steps > 0 else max(1, steps)


def run_loop(name: str, examples: Sequence, step_fn: Callable[[List], float], *, ctx, trainer, tokenizer,
             output_dir: str, per_device: int, accum: int, epochs: float, max_steps: int = -1,
             logging_steps: int = 10, save_steps: int = 0, seed: int = 0, save_total_limit: int = 1) -> dict:
    n = len(examples)
    total = plan_steps(n, ctx.world, per_device, accum, epochs, max_steps)
    start = 0
    ck = latest_checkpoint(output_dir)
    if ck is not None:
        import json
        from ..models.hf_io import load_weights
        if hasattr(trainer, "load_checkpoint"):
            trainer.load_checkpoint(ck)
        else:
            load_weights(trainer.w, ck)
        start = json.load(open(os.path.join(ck, "trainer_state.json"))).get("global_step", 0)
        opt_f = os.path.join(ck, f"optimizer-rank{ctx.rank}.pt")
        if os.path.exists(opt_f):
            trainer.opt.load_state_dict(torch.load(opt_f, map_location="cpu"))
        log.info("resumed", checkpoint=ck, step=start)
    order = list(range(n))
    per_rank_step = per_device * accum
    history = []
    hb = None
    if ctx.world > 1:
        from ..parallel.health import Heartbeat
        store = _default_store()
        if store is not None:
            hb = Heartbeat(store, ctx.rank, ctx.world, timeout_s=float(os.environ.get("KORE_HEARTBEAT_S", "600")))
    for step in range(start, total):
        if hb is not None and step > start:
            hb.wait_peers(step - 1)              # a lost peer stops us between steps, not inside a collective
        epoch = (step * per_rank_step * ctx.world) // max(1, n)
        rng = random.Random(seed + epoch)
        perm = order[:]
        rng.shuffle(perm)
        base = (step * per_rank_step * ctx.world) % max(1, n)
        idx = [perm[(base + ctx.rank + ctx.world * j) % n] for j in range(per_rank_step)]
        loss = step_fn([examples[i] for i in idx])
        history.append(loss)
        if hb is not None:
            hb.beat(step)
        if ctx.is_main and ((step + 1) % max(1, logging_steps) == 0 or step == total - 1):
            log.event(f"{name}_step", step=step + 1, loss=round(loss, 5), lr=trainer.opt.current_lr(),
                      epoch=epoch)
        if save_steps and (step + 1) % save_steps == 0 and step + 1 < total:
            d = os.path.join(output_dir, f"checkpoint-{step + 1}")
            full = trainer.full_weights() if hasattr(trainer, "full_weights") else trainer.w   # collective
            if ctx.is_main:
                save_pretrained(full, d, tokenizer, keep_last=save_total_limit,
                                trainer_state={"global_step": step + 1})
            ctx.barrier()
            torch.save(trainer.opt.state_dict(), os.path.join(d, f"optimizer-rank{ctx.rank}.pt"))
    full = trainer.full_weights() if hasattr(trainer, "full_weights") else trainer.w
    if ctx.is_main:
        save_pretrained(full, output_dir, tokenizer)
    if hb is not None:
        hb.leave()
    ctx.barrier()
    return {"output_dir": output_dir, "steps": total, "history": history}


def _default_store():
    try:
        import torch.distributed as dist
        from torch.distributed import distributed_c10d as c10d
        return c10d._get_default_store() if dist.is_initialized() else None
    except Exception:  # noqa: BLE001 - no store: run without heartbeats
        return None
