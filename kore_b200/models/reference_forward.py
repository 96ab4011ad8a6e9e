"""Plain-autograd fp32 forward of a Qwen3 dense model over packed sequences.

This is the oracle the explicit engine (and every kernel it calls) is checked
against: same weights, same batch, every op from ``kore_b200.ops.reference``
in fp32 with torch autograd for the gradients."""
from __future__ import annotations

from typing import List

import torch

from ..ops import reference as ref
from .qwen3 import Qwen3Weights


def leaf_buffers(w: Qwen3Weights) -> List[torch.Tensor]:
    return [b.detach().float().clone().requires_grad_(True) for b in w.bufs]


def forward_logprobs(w: Qwen3Weights, bufs: List[torch.Tensor], batch, temperature: float = 1.0):
    cfg = w.cfg
    hq, hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    eps = cfg.rms_norm_eps
    cos, sin = ref.rope_tables(cfg.max_position_embeddings, D, cfg.rope_theta, bufs[0].device)
    V = [lay.views(b) for lay, b in zip(w.layouts, bufs)]
    x = V[0]["embed"][batch.ids]
    T = x.shape[0]
    qd, kd = hq * D, hkv * D
    for u in range(1, len(bufs) - 1):
        W = V[u]
        hn = ref.rmsnorm(x, W["ln1"], eps)
        qkv = hn @ W["qkv"].t()
        qk = ref.qk_norm_rope(qkv, W["q_norm"], W["k_norm"], batch.pos, cos, sin, hq, hkv, eps)
        q = qk[:, :qd].reshape(T, hq, D)
        k = qk[:, qd:].reshape(T, hkv, D)
        v = qkv[:, qd + kd:].reshape(T, hkv, D)
        o = ref.causal_attention(q, k, v, cu_seqlens=batch.cu_seqlens)
        x = x + o.reshape(T, qd) @ W["o"].t()
        hn2 = ref.rmsnorm(x, W["ln2"], eps)
        if w.layouts[u].kind == "moe_layer":
            x = x + moe_block(cfg, W, hn2)
        else:
            a = ref.swiglu(hn2 @ W["gate_up"].t())
            x = x + a @ W["down"].t()
    Wh = V[-1]
    hn = ref.rmsnorm(x, Wh["norm"], eps)
    lm = V[0]["embed"] if cfg.tie_word_embeddings else Wh["lm_head"]
    logits = hn @ lm.t()
    lp, ent, _ = ref.token_logprobs(logits, batch.targets, temperature)
    lp = torch.where(batch.targets >= 0, lp, torch.zeros_like(lp))
    return lp, ent


def moe_block(cfg, W, h):
    """Qwen3-MoE sparse block: softmax router, top-k, renormalised weights,
    SwiGLU experts, weighted sum (dense loop over experts; oracle only)."""
    logits = h @ W["router"].t()
    probs = torch.softmax(logits.float(), -1)
    wts, idx = probs.topk(cfg.num_experts_per_tok, -1)
    if cfg.norm_topk_prob:
        wts = wts / wts.sum(-1, keepdim=True)
    out = torch.zeros_like(h, dtype=torch.float32)
    for e in range(cfg.num_experts):
        sel = (idx == e)
        rows = sel.any(-1)
        if not rows.any():
            continue
        we = (wts * sel).sum(-1)[rows]
        a = ref.swiglu(h[rows] @ W["experts_gate_up"][e].t())
        out = out.index_add(0, rows.nonzero()[:, 0], (a @ W["experts_down"][e].t()).float() * we[:, None])
    return out.to(h.dtype)
