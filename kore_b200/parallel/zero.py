"""Sharded data parallelism for the flat-unit engine (ZeRO-2 style).

Every rank keeps the full bf16 parameters and accumulates full gradients for
its micro-batches; at the step boundary each unit's gradient is
reduce-scattered, the rank updates only its 1/world shard (fp32 moments and
optional fp32 master live only for the shard), and the updated bf16 shard is
all-gathered back into every rank's full parameter buffer.

Per step and unit that moves the same bytes as one all-reduce, while the
optimizer state and AdamW work drop by ``world``. Two data planes:

* ``comm="nccl"``: NCCL reduce-scatter / all-gather (the baseline);
* ``comm="fused"``: the native peer-memory kernel that fuses the
  reduce-scatter with the bf16->fp32 cast, the global-norm clip and the AdamW
  update (``kore_b200.parallel.fused_rs_adamw``), then broadcasts the shard
  with NVLink stores.

Reference parity: FSDP SHARD_GRAD_OP / FULL_SHARD via accelerate
(kore/policy/configs.py:580-651, kore/policy/grpo.py:1562-1625). With 180 GB of
HBM per GPU a 14B model's full bf16 weights stay resident, so no per-layer
re-gather is needed inside the step.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..engine.optimizer import lr_lambda_factory
from .dist import DistContext


class ShardedAdamW:
    def __init__(self, weights, engine, ctx: DistContext, lr: float = 1e-5, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, max_grad_norm: float = 0.0,
                 master: str = "fp32", schedule: str = "constant", warmup_steps: int = 0,
                 total_steps: int = 1, seed: int = 0, comm: str = "nccl"):
        self.w, self.eng, self.ctx = weights, engine, ctx
        self.lr, (self.b1, self.b2), self.eps, self.wd = lr, betas, eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.lr_fn = lr_lambda_factory(schedule, warmup_steps, total_steps)
        self.step_count = 0
        self.seed = seed
        self.comm = comm
        W, r = ctx.world, ctx.rank
        dev = weights.device
        self.shard_len = []
        self.m, self.v, self.master, self.gshard = {}, {}, {}, {}
        for u in range(weights.num_units):
            n = weights.bufs[u].numel()
            assert n % W == 0, "weights must be padded to a multiple of world"
            s = n // W
            self.shard_len.append(s)
            self.m[u] = torch.zeros(s, dtype=torch.float32, device=dev)
            self.v[u] = torch.zeros(s, dtype=torch.float32, device=dev)
            if master == "fp32":
                self.master[u] = weights.bufs[u][r * s:(r + 1) * s].float()
            if comm != "fused":   # the fused path reads peers' gradients in place
                self.gshard[u] = torch.empty(s, dtype=engine.grad_dtype, device=dev)
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.last_sumsq: Optional[torch.Tensor] = None
        self.local = None      # ListAdamW over expert-parallel expert weights, if any

    def current_lr(self) -> float:
        return self.lr * self.lr_fn(self.step_count)

    def reduce_scatter_unit(self, u: int, async_op: bool = False):
        if self.ctx.backend != "nccl":   # gloo has no reduce-scatter: all-reduce + slice
            g = self.eng.grads[u]
            dist.all_reduce(g, group=self.ctx.group)
            s = self.shard_len[u]
            self.gshard[u].copy_(g[self.ctx.rank * s:(self.ctx.rank + 1) * s])
            return None
        return dist.reduce_scatter_tensor(self.gshard[u], self.eng.grads[u], op=dist.ReduceOp.SUM,
                                          group=self.ctx.group, async_op=async_op)

    def all_gather_unit(self, u: int) -> None:
        s = self.shard_len[u]
        r = self.ctx.rank
        if self.ctx.backend != "nccl":
            parts = [torch.empty_like(self.w.bufs[u][:s]) for _ in range(self.ctx.world)]
            dist.all_gather(parts, self.w.bufs[u][r * s:(r + 1) * s].clone(), group=self.ctx.group)
            self.w.bufs[u].copy_(torch.cat(parts))
            return
        # in place: NCCL accepts send == recv + rank * count
        dist.all_gather_into_tensor(self.w.bufs[u], self.w.bufs[u][r * s:(r + 1) * s],
                                    group=self.ctx.group)

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, scattered: bool = False) -> None:
        W, r = self.ctx.world, self.ctx.rank
        if not scattered:
            for u in range(self.w.num_units):
                self.reduce_scatter_unit(u)
        sq = None
        if self.max_grad_norm and self.max_grad_norm > 0:
            self._sumsq.zero_()
            for u in range(self.w.num_units):
                ops.sumsq(self.gshard[u], self._sumsq)
            if self.local is not None:        # disjoint across ranks: add before the reduce
                self.local.add_sumsq(self._sumsq)
            dist.all_reduce(self._sumsq, group=self.ctx.group)
            sq = self._sumsq
            self.last_sumsq = sq
        if self.local is not None:
            self.local.step(sq, float(self.max_grad_norm or 0.0))
        lr = self.current_lr()
        self.step_count += 1
        for u in range(self.w.num_units):
            s = self.shard_len[u]
            pshard = self.w.bufs[u][r * s:(r + 1) * s]
            ops.adamw_step(pshard, self.gshard[u], self.m[u], self.v[u], lr=lr, b1=self.b1,
                           b2=self.b2, eps=self.eps, wd=self.wd, step=self.step_count,
                           grad_scale=grad_scale, master=self.master.get(u), sumsq_buf=sq,
                           max_norm=self.max_grad_norm,
                           seed=self.seed * 7919 + self.step_count * 104729 + u * 31 + r)
            self.all_gather_unit(u)

    def grad_norm(self) -> float:
        return float(self.last_sumsq.sqrt()) if self.last_sumsq is not None else float("nan")

    def state_dict(self) -> dict:
        """This rank's optimizer shard (moments, master, step, expert-local state)."""
        sd = {"step": self.step_count, "rank": self.ctx.rank, "world": self.ctx.world,
              "m": {u: t.cpu() for u, t in self.m.items()}, "v": {u: t.cpu() for u, t in self.v.items()},
              "master": {u: t.cpu() for u, t in self.master.items()}}
        if self.local is not None and hasattr(self.local, "state_dict"):
            sd["local"] = self.local.state_dict()
        return sd

    def load_state_dict(self, sd: dict) -> None:
        if sd.get("world", self.ctx.world) != self.ctx.world:
            raise ValueError(f"optimizer shard saved at world {sd['world']}, loading at {self.ctx.world}")
        self.step_count = int(sd["step"])
        for k in ("m", "v", "master"):
            for u, t in sd.get(k, {}).items():
                getattr(self, k)[int(u)].copy_(t)
        if "local" in sd and self.local is not None:
            self.local.load_state_dict(sd["local"])


class FusedShardedAdamW(ShardedAdamW):
    """ZeRO-2 step on the symmetric peer-memory heap with fused kernels:

    device barrier -> (with clipping) per unit: the sum of squares of this
    rank's gradient shard, reduced over peers with NVLink P2P loads -> device
    all-reduce of the norm -> per unit: ONE kernel that reduce-scatters the
    bf16 gradients (P2P loads from every peer, fp32 sum), applies the clipped
    AdamW update to the fp32 shard state and all-gathers the result (P2P
    stores of the new bf16 parameters into every peer) -> device barrier.
    No NCCL call, no host sync, and no gradient-shard buffer.
    Parameters and gradients must live in ``heap`` (see
    :meth:`CausalLMTrainer` with ``comm="fused"``)."""

    def __init__(self, weights, engine, ctx, heap, **kw):
        kw["comm"] = "fused"
        super().__init__(weights, engine, ctx, **kw)
        self.heap = heap
        dev = weights.device
        self._local = torch.zeros(1, dtype=torch.float32, device=dev)
        self.p_off = [heap.offset_of(b) for b in weights.bufs]
        self.g_off = [heap.offset_of(g) for g in engine.grads]

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, scattered: bool = False) -> None:
        from .. import ops
        C = ops.native()
        h = self.heap
        h.barrier()                                   # every rank's gradients are final
        sq = None
        if self.max_grad_norm and self.max_grad_norm > 0:
            self._local.zero_()
            for u in range(self.w.num_units):
                C.symm_rs_sumsq(h.id, self.g_off[u], self.shard_len[u], None, self._local, float(grad_scale))
            if self.local is not None:
                self.local.add_sumsq(self._local)
            C.symm_scalar_allreduce(h.id, 0, h.next_epoch(), self._local, self._sumsq)
            sq = self._sumsq
            self.last_sumsq = sq
        lr = self.current_lr()
        self.step_count += 1
        for u in range(self.w.num_units):
            C.symm_adamw_bcast(h.id, self.p_off[u], self.g_off[u], self.shard_len[u], float(grad_scale),
                               self.master.get(u),
                               self.m[u], self.v[u], lr, self.b1, self.b2, self.eps, self.wd,
                               self.step_count, sq, float(self.max_grad_norm or 0.0),
                               self.seed * 7919 + self.step_count * 104729 + u * 31 + self.ctx.rank)
        if self.local is not None:
            self.local.step(sq, float(self.max_grad_norm or 0.0))
        h.barrier()                                   # every rank received all parameter shards
