"""AdamW over the flat per-unit buffers, plus the LR schedules.

One fused kernel launch per unit updates params (+ optional fp32 master),
first/second moments. Global grad-norm clipping is done without a host sync:
a reduction kernel accumulates sum(g^2) over all units into one device
scalar, and the AdamW kernel derives the clip factor from it.

``master="fp32"`` keeps an fp32 master copy (exact fp32 AdamW);
``master="none"`` keeps bf16 params and rounds each update stochastically
(unbiased), which saves 4 bytes/param — what lets a 14B model with fp32
moments train on one 180 GB GPU.

Reference parity: AdamW + LambdaLR warmup then constant/linear/cosine
(kore/policy/grpo.py:862-890) and grad-norm clipping
(kore/policy/grpo.py:2299).
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch

from .. import ops


def lr_lambda_factory(schedule: str, warmup_steps: int, total_steps: int):
    """Multiplier on the base LR at optimizer step ``step`` (0-based), as the
    reference's LambdaLR: linear warmup, then constant / linear / cosine decay."""
    schedule = (schedule or "constant").lower()

    def f(step: int) -> float:
        if warmup_steps > 0 and step < warmup_steps:
            return float(step + 1) / float(warmup_steps)
        if schedule in ("constant", "constant_with_warmup"):
            return 1.0
        span = max(1, total_steps - warmup_steps)
        prog = min(1.0, max(0.0, (step - warmup_steps) / span))
        if schedule == "linear":
            return max(0.0, 1.0 - prog)
        if schedule == "cosine":
            return 0.5 * (1.0 + math.cos(math.pi * prog))
        raise ValueError(f"unknown lr schedule {schedule!r}")

    return f


class AdamW:
    def __init__(self, weights, engine, lr: float = 1e-5, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_grad_norm: float = 0.0, master: str = "auto",
                 schedule: str = "constant", warmup_steps: int = 0, total_steps: int = 1,
                 units: Optional[List[int]] = None, seed: int = 0):
        self.w = weights
        self.eng = engine
        self.lr = lr
        self.b1, self.b2 = betas
        self.eps = eps
        self.wd = weight_decay
        self.max_grad_norm = max_grad_norm
        self.step_count = 0
        self.seed = seed
        self.lr_fn = lr_lambda_factory(schedule, warmup_steps, total_steps)
        self.units = units if units is not None else list(range(weights.num_units))
        dev = weights.device
        if master == "auto":
            master = "fp32" if weights.dtype != torch.float32 else "none"
        self.master_mode = master
        self.m = {}
        self.v = {}
        self.master = {}
        for u in self.units:
            n = weights.bufs[u].numel()
            self.m[u] = torch.zeros(n, dtype=torch.float32, device=dev)
            self.v[u] = torch.zeros(n, dtype=torch.float32, device=dev)
            if master == "fp32" and weights.dtype != torch.float32:
                self.master[u] = weights.bufs[u].float()
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.last_grad_norm: Optional[torch.Tensor] = None

    def current_lr(self) -> float:
        return self.lr * self.lr_fn(self.step_count)

    def grad_sumsq(self) -> torch.Tensor:
        self._sumsq.zero_()
        for u in self.units:
            ops.sumsq(self.eng.grads[u], self._sumsq)
        return self._sumsq

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, sumsq: Optional[torch.Tensor] = None) -> None:
        """Apply one update. ``sumsq`` lets a sharded caller pass the globally
        all-reduced sum of squares; otherwise it is computed locally."""
        lr = self.current_lr()
        self.step_count += 1
        sq = None
        if self.max_grad_norm and self.max_grad_norm > 0:
            sq = sumsq if sumsq is not None else self.grad_sumsq()
            self.last_grad_norm = sq
        for u in self.units:
            p = self.w.bufs[u]
            if p.dtype == torch.float32:
                ops.adamw_step_f32(p, self.eng.grads[u], self.m[u], self.v[u], lr=lr, b1=self.b1,
                                   b2=self.b2, eps=self.eps, wd=self.wd, step=self.step_count,
                                   grad_scale=grad_scale, sumsq_buf=sq,
                                   max_norm=self.max_grad_norm)
                continue
            ops.adamw_step(p, self.eng.grads[u], self.m[u], self.v[u], lr=lr, b1=self.b1,
                           b2=self.b2, eps=self.eps, wd=self.wd, step=self.step_count,
                           grad_scale=grad_scale, master=self.master.get(u), sumsq_buf=sq,
                           max_norm=self.max_grad_norm,
                           seed=self.seed * 7919 + self.step_count * 104729 + u)

    def grad_norm(self) -> float:
        if self.last_grad_norm is None:
            return float(self.grad_sumsq().sqrt())
        return float(self.last_grad_norm.sqrt())

    def state_dict(self) -> dict:
        return {"step": self.step_count, "m": {u: t.cpu() for u, t in self.m.items()},
                "v": {u: t.cpu() for u, t in self.v.items()},
                "master": {u: t.cpu() for u, t in self.master.items()}}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        for u, t in sd["m"].items():
            self.m[int(u)].copy_(t)
        for u, t in sd["v"].items():
            self.v[int(u)].copy_(t)
        for u, t in sd.get("master", {}).items():
            self.master[int(u)].copy_(t)


class ListAdamW:
    """AdamW over an explicit {key: (param, grad)} set (expert-parallel expert
    weights, which are local to their rank and never sharded)."""

    def __init__(self, params: dict, grads: dict, lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, master: str = "fp32", schedule: str = "constant",
                 warmup_steps: int = 0, total_steps: int = 1, seed: int = 0):
        self.p, self.g = params, grads
        self.lr, (self.b1, self.b2), self.eps, self.wd = lr, betas, eps, weight_decay
        self.lr_fn = lr_lambda_factory(schedule, warmup_steps, total_steps)
        self.step_count = 0
        self.seed = seed
        self.m = {k: torch.zeros(v.numel(), dtype=torch.float32, device=v.device) for k, v in params.items()}
        self.v = {k: torch.zeros(v.numel(), dtype=torch.float32, device=v.device) for k, v in params.items()}
        self.master = ({k: v.float().clone() for k, v in params.items()}
                       if master == "fp32" and any(v.dtype != torch.float32 for v in params.values()) else {})

    def add_sumsq(self, acc: torch.Tensor) -> None:
        for g in self.g.values():
            ops.sumsq(g, acc)

    @torch.no_grad()
    def step(self, sumsq: Optional[torch.Tensor] = None, max_norm: float = 0.0) -> None:
        lr = self.lr * self.lr_fn(self.step_count)
        self.step_count += 1
        for k, p in self.p.items():
            if p.dtype == torch.float32:
                ops.adamw_step_f32(p, self.g[k], self.m[k], self.v[k], lr=lr, b1=self.b1, b2=self.b2,
                                   eps=self.eps, wd=self.wd, step=self.step_count, sumsq_buf=sumsq,
                                   max_norm=max_norm)
            else:
                ops.adamw_step(p, self.g[k], self.m[k], self.v[k], lr=lr, b1=self.b1, b2=self.b2, eps=self.eps,
                               wd=self.wd, step=self.step_count, master=self.master.get(k), sumsq_buf=sumsq,
                               max_norm=max_norm, seed=self.seed * 31 + self.step_count * 7 + int(k))
