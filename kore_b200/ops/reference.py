"""Plain PyTorch (fp32-math) definitions of every hot op.

These are the oracles the native kernels are tested against, and the CPU
implementation used by CPU tests and gloo runs. They follow the HF Qwen3
definitions (RMSNorm, rotate-half RoPE, SiLU-gated MLP) that the reference's
trainers run through transformers (kore/policy/configs.py:550-567).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r * w.float()).to(x.dtype)


def rope_tables(max_pos: int, head_dim: int, theta: float, device=None):
    """cos/sin tables [max_pos, head_dim/2] in fp32 (rotate-half convention)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return f.cos().float().to(device), f.sin().float().to(device)


def apply_rope(x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """x: [T, H, D]; rotate-half RoPE in fp32."""
    d2 = x.shape[-1] // 2
    c = cos[pos.long()].unsqueeze(1)
    s = sin[pos.long()].unsqueeze(1)
    xf = x.float()
    x1, x2 = xf[..., :d2], xf[..., d2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def qk_norm_rope(qkv, qw, kw, pos, cos, sin, hq, hkv, eps):
    T = qkv.shape[0]
    D = qkv.shape[1] // (hq + 2 * hkv)
    q = qkv[:, : hq * D].reshape(T, hq, D)
    k = qkv[:, hq * D : (hq + hkv) * D].reshape(T, hkv, D)
    q = apply_rope(rmsnorm(q, qw, eps), pos, cos, sin)
    k = apply_rope(rmsnorm(k, kw, eps), pos, cos, sin)
    return torch.cat([q.reshape(T, -1), k.reshape(T, -1)], dim=1)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    f = gu.shape[-1] // 2
    g, u = gu[..., :f].float(), gu[..., f:].float()
    return (F.silu(g) * u).to(gu.dtype)


def causal_attention(q, k, v, scale=None, cu_seqlens=None):
    """q: [T, Hq, D], k/v: [T, Hkv, D] packed; causal within each sequence."""
    T, hq, D = q.shape
    hkv = k.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    rep = hq // hkv
    if cu_seqlens is None:
        cu = [0, T]
    else:
        cu = [int(c) for c in cu_seqlens.tolist()]
    out = torch.empty_like(q)
    for a, b in zip(cu[:-1], cu[1:]):
        qs = q[a:b].float().transpose(0, 1)
        ks = k[a:b].float().repeat_interleave(rep, 1).transpose(0, 1)
        vs = v[a:b].float().repeat_interleave(rep, 1).transpose(0, 1)
        s = (qs @ ks.transpose(-1, -2)) * scale
        n = b - a
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
        p = s.softmax(-1)
        out[a:b] = (p @ vs).transpose(0, 1).to(q.dtype)
    return out


def token_logprobs(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0):
    """Per-token log p(target) and entropy over the full vocab, fp32."""
    z = logits.float() / temperature
    lse = torch.logsumexp(z, -1)
    lp = z.gather(-1, targets.long().clamp_min(0).unsqueeze(-1)).squeeze(-1) - lse
    p = torch.softmax(z, -1)
    ent = lse - (p * z).sum(-1)
    return lp, ent, lse
