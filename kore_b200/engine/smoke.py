"""Tiny end-to-end forward+backward of the flagship training engine (used by
``__graft_entry__.smoke``): a 2-layer Qwen3-architecture model in bf16 on the
GPU, one packed micro-batch of two sequences, SFT loss, one AdamW step."""
from __future__ import annotations

import torch

from ..models import Qwen3Config, Qwen3Weights
from .qwen3_engine import Batch, Qwen3Engine
from .optimizer import AdamW


def smoke_config() -> Qwen3Config:
    return Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=128, max_position_embeddings=1024)


def run_smoke(device="cuda:0") -> dict:
    torch.cuda.set_device(torch.device(device))
    cfg = smoke_config()
    w = Qwen3Weights(cfg, device=device, dtype=torch.bfloat16, seed=0)
    eng = Qwen3Engine(w)
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (200, 120)]
    b = Batch.from_sequences(seqs, device=device)
    lp0, _ = eng.token_logprobs(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=eng.sft_coef(b))
    opt = AdamW(w, eng, lr=1e-3)
    opt.step()
    lp1, _ = eng.token_logprobs(b)
    valid = b.targets >= 0
    before = -lp0[valid].mean().item()
    after = -lp1[valid].mean().item()
    torch.cuda.synchronize()
    assert torch.isfinite(torch.tensor([before, after])).all(), (before, after)
    assert after < before, f"loss did not decrease: {before} -> {after}"
    return {"loss_before": before, "loss_after": after}
