"""Supervised fine-tuning (repair-weighted, completion-only) on the explicit engine.

Chat rows are rendered in Qwen ChatML; with ``assistant_only_loss`` the
loss covers only assistant tokens (mask from the renderer); repair rows are
up-sampled by ``repair_loss_weight``; rows longer than ``max_seq_length`` are
dropped. Steps pack ``per_device_train_batch_size * gradient_accumulation_steps``
rows per rank into token-budget micro-batches (varlen attention, no padding).

Entry point: ``python -m kore_b200.policy.sft cfg.json`` (same JSON schema as
the reference, kore/policy/sft.py:246-465).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path
from typing import Optional

import torch

from ..data.datasets import load_sft_rows
from ..data.tokenizer import load_tokenizer, render_chat
from ..models.hf_io import load_pretrained_or_init
from ..obs import configure, get_logger
from ..parallel.dist import init_distributed
from ._loop import plan_steps, run_loop
from .configs import parallel_kwargs as _parallel_kwargs
from .configs import SFTConfig, sft_config_from_dict

log = get_logger("policy.sft")


def tokenize_chat_rows(rows, tok, max_len: int, assistant_only: bool = True):
    out, dropped = [], 0
    for r in rows:
        ids, mask = render_chat(tok, r["messages"])
        if max_len and len(ids) > max_len:
            dropped += 1
            continue
        lab = mask if assistant_only else [1] * len(ids)
        if sum(lab[1:]) == 0:
            continue
        out.append((ids, lab))
    return out, dropped


def train_sft(config: SFTConfig, dataset_path: Optional[str] = None, *, model_cfg=None, tokenizer=None,
              weights=None) -> dict:
    from ..engine.trainer import CausalLMTrainer
    ctx = init_distributed()
    configure(config.output_dir)
    tok = tokenizer or load_tokenizer(config.model_id)
    rows = load_sft_rows(dataset_path or config.dataset_path, config.repair_loss_weight)
    ex, dropped = tokenize_chat_rows(rows, tok, config.max_seq_length, config.assistant_only_loss)
    if ctx.is_main:
        log.info("sft data", rows=len(rows), kept=len(ex), dropped_overlong=dropped)
    w = weights or load_pretrained_or_init(config.model_id, ctx, model_cfg=model_cfg, bf16=config.bf16,
                                           seed=config.seed)
    total = plan_steps(len(ex), ctx.world, config.per_device_train_batch_size,
                       config.gradient_accumulation_steps, config.num_train_epochs, config.max_steps)
    tr = CausalLMTrainer(w.cfg, ctx, lr=config.learning_rate, weight_decay=config.weight_decay,
                         max_grad_norm=config.max_grad_norm, seed=config.seed,
                         schedule=config.lr_scheduler_type, warmup_steps=int(config.warmup_ratio * total),
                         total_steps=total, weights=w, **_parallel_kwargs(config, ctx.world))
    tr.eng.save_attention = config.save_attention
    budget = config.micro_batch_tokens or max(config.max_seq_length, 8192)
    step_fn = lambda exs: tr.train_step_sequences([e[0] for e in exs], [e[1] for e in exs],
                                                  micro_tokens=budget)
    return run_loop("sft", ex, step_fn, ctx=ctx, trainer=tr, tokenizer=tok, output_dir=config.output_dir,
                    per_device=config.per_device_train_batch_size, accum=config.gradient_accumulation_steps,
                    epochs=config.num_train_epochs, max_steps=config.max_steps,
                    logging_steps=config.logging_steps, save_steps=config.save_steps, seed=config.seed,
                    save_total_limit=config.save_total_limit)


def _main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print("usage: python -m kore_b200.policy.sft <config.json>", file=sys.stderr)
        return 2
    raw = json.loads(Path(argv[0]).read_text())
    raw.setdefault("distributed", True)
    cfg, path = sft_config_from_dict(raw)
    print(f"[sft] -> {train_sft(cfg, path)['output_dir']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
