"""WiSE-FT weight soup: theta = (1 - alpha) * base + alpha * kore, with an
alpha sweep guarded by a retention gate and a base-ward fallback
(reference: kore/policy/soup.py:20-120). Interpolation runs unit by unit on
the flat buffers (one fused lerp per unit)."""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch

from ..models.hf_io import from_pretrained, save_pretrained
from ..models.qwen3 import Qwen3Weights
from .configs import SoupConfig


@torch.no_grad()
def interpolate(base: Qwen3Weights, kore: Qwen3Weights, alpha: float) -> Qwen3Weights:
    if base.cfg.to_dict() != kore.cfg.to_dict():
        raise ValueError("soup: architectures differ")
    out = base.clone()
    for o, k in zip(out.bufs, kore.bufs):
        o.lerp_(k.to(o.dtype), float(alpha))
    return out


def sweep_alphas(base, kore, alphas: Sequence[float], retention_fn: Callable[[Qwen3Weights], float],
                 base_score: float, epsilon: float = 0.005):
    """Largest alpha whose retention score regresses by at most ``epsilon`` from
    the base; walks toward the base (smaller alpha) when every alpha fails."""
    best = None
    for a in sorted(alphas, reverse=True):
        w = interpolate(base, kore, a)
        s = retention_fn(w)
        if s >= base_score - epsilon:
            return a, w, s
        best = best or (a, w, s)
    a = min(alphas) / 2.0
    w = interpolate(base, kore, a)
    return a, w, retention_fn(w)


def build_soup(config: SoupConfig, retention_fn: Optional[Callable] = None, device="cpu") -> dict:
    base = from_pretrained(config.base_model_id, device=device)
    kore = from_pretrained(config.kore_checkpoint, device=device)
    if retention_fn is None:
        a = max(config.alphas)
        w = interpolate(base, kore, a)
        score = None
    else:
        a, w, score = sweep_alphas(base, kore, config.alphas, retention_fn, retention_fn(base), config.epsilon)
    save_pretrained(w, config.output_dir)
    return {"alpha": a, "retention": score, "output_dir": config.output_dir}
