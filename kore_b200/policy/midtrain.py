"""Continued pre-training on a text corpus (``{"text"}`` JSONL).

Documents are tokenized, terminated with EOS and packed back to back into
``max_seq_length``-token windows; attention is causal within each document
(varlen packing, so no cross-document attention and no padding). Loss on
every token. Entry: ``python -m kore_b200.policy.midtrain cfg.json``
(reference: kore/policy/midtrain.py:38-269).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

from ..data.datasets import load_text_rows
from ..data.tokenizer import eos_ids, load_tokenizer
from ..models.hf_io import load_pretrained_or_init
from ..obs import configure, get_logger
from ..parallel.dist import init_distributed
from ._loop import plan_steps, run_loop
from .configs import parallel_kwargs as _parallel_kwargs
from .configs import MidTrainConfig, midtrain_config_from_dict

log = get_logger("policy.midtrain")


def pack_documents(texts, tok, max_len: int):
    """Greedy packing into windows; a window is a list of documents (id lists)."""
    eos = (eos_ids(tok) or [0])[0]
    windows, cur, n = [], [], 0
    for t in texts:
        ids = list(tok.encode(t)) + [eos]
        while ids:
            room = max_len - n
            piece, ids = ids[:room], ids[room:]
            cur.append(piece)
            n += len(piece)
            if n >= max_len:
                windows.append(cur)
                cur, n = [], 0
    if cur:
        windows.append(cur)
    return windows


def train_midtrain(config: MidTrainConfig, corpus_path=None, *, model_cfg=None, tokenizer=None, weights=None):
    from ..engine.trainer import CausalLMTrainer
    ctx = init_distributed()
    configure(config.output_dir)
    tok = tokenizer or load_tokenizer(config.model_id)
    windows = pack_documents(load_text_rows(corpus_path or config.corpus_path), tok, config.max_seq_length)
    w = weights or load_pretrained_or_init(config.model_id, ctx, model_cfg=model_cfg, bf16=config.bf16,
                                           seed=config.seed)
    total = plan_steps(len(windows), ctx.world, config.per_device_train_batch_size,
                       config.gradient_accumulation_steps, config.num_train_epochs, config.max_steps)
    tr = CausalLMTrainer(w.cfg, ctx, lr=config.learning_rate, weight_decay=config.weight_decay,
                         max_grad_norm=config.max_grad_norm, seed=config.seed,
                         schedule=config.lr_scheduler_type, warmup_steps=int(config.warmup_ratio * total),
                         total_steps=total, weights=w, **_parallel_kwargs(config, ctx.world))

    def step_fn(wins):
        seqs = [d for win in wins for d in win]
        masks = [[1] * len(d) for d in seqs]
        return tr.train_step_sequences(seqs, masks, micro_tokens=config.max_seq_length)

    return run_loop("midtrain", windows, step_fn, ctx=ctx, trainer=tr, tokenizer=tok,
                    output_dir=config.output_dir, per_device=config.per_device_train_batch_size,
                    accum=config.gradient_accumulation_steps, epochs=config.num_train_epochs,
                    max_steps=config.max_steps, logging_steps=config.logging_steps,
                    save_steps=config.save_steps, seed=config.seed, save_total_limit=config.save_total_limit)


def _main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print("usage: python -m kore_b200.policy.midtrain <config.json>", file=sys.stderr)
        return 2
    raw = json.loads(Path(argv[0]).read_text())
    raw.setdefault("distributed", True)
    cfg = midtrain_config_from_dict(raw)
    print(f"[midtrain] -> {train_midtrain(cfg)['output_dir']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
