"""NVLink SHARP data plane for the ZeRO-2 step (``comm="nvls"``).

Parameters and gradients of all units live in two flat buffers allocated with
torch's symmetric memory and bound to an NVLink multicast object (one
physical copy per GPU, one multicast address for all). The optimizer step
(:class:`NVLSShardedAdamW`) reads, for each rank's shard, the sum of every
rank's gradients straight out of the switch (``multimem.ld_reduce``) and
writes the updated parameters to every rank with one multicast store
(``multimem.st``); see ``csrc/nvls_sm100.cu``. Flag barriers of a small
symmetric heap order the step against the ranks' backward passes and next
forward passes.

``NVLSBuffers.available`` is False when the platform has no multicast support
(no NVSwitch, or a driver / container without it); the trainer then refuses
``comm="nvls"`` instead of silently switching data planes.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch

from .dist import DistContext
from .zero import ShardedAdamW


class NVLSUnavailable(RuntimeError):
    pass


class NVLSBuffers:
    ALIGN = 256          # bytes

    def __init__(self, ctx: DistContext, elems: int, dtype=torch.bfloat16):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.ctx, self.dtype = ctx, dtype
        esz = torch.empty((), dtype=dtype).element_size()
        self.elems = int(elems)
        group = ctx.group if ctx.group is not None else dist.group.WORLD
        self.buf = symm.empty(self.elems, dtype=dtype, device=ctx.device)
        self.handle = symm.rendezvous(self.buf, group)
        self.mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if self.mc == 0:
            raise NVLSUnavailable("no NVLink multicast object for this group (no NVLS on this platform)")
        self.esz = esz
        self.next = 0

    def alloc(self, n: int, dtype=None) -> torch.Tensor:
        if dtype is not None and dtype != self.dtype:
            raise ValueError("NVLS buffers hold one dtype")
        per = self.ALIGN // self.esz
        start = (self.next + per - 1) // per * per
        if start + n > self.elems:
            raise MemoryError("NVLS buffer exhausted")
        self.next = start + int(n)
        return self.buf[start:start + int(n)]

    def mc_addr(self, t: torch.Tensor, elem: int = 0) -> int:
        """Multicast address of element ``elem`` of ``t`` (a view of the buffer)."""
        off = (t.data_ptr() - self.buf.data_ptr()) // self.esz + int(elem)
        return self.mc + off * self.esz


class NVLSShardedAdamW(ShardedAdamW):
    """ZeRO-2 step through the switch: barrier -> (clipping) switch-reduced
    sum of squares of each shard, device scalar all-reduce -> per unit one
    kernel: switch-reduced gradient shard, clipped AdamW on the fp32 shard
    state, multicast store of the new bf16 parameters -> barrier."""

    def __init__(self, weights, engine, ctx, pbuf: NVLSBuffers, gbuf: NVLSBuffers, heap, **kw):
        kw["comm"] = "fused"
        super().__init__(weights, engine, ctx, **kw)
        self.pbuf, self.gbuf, self.heap = pbuf, gbuf, heap
        self._local = torch.zeros(1, dtype=torch.float32, device=weights.device)

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, scattered: bool = False) -> None:
        from .. import ops
        C = ops.native()
        h, r = self.heap, self.ctx.rank
        h.barrier()                                   # every rank's gradients are final
        sq = None
        if self.max_grad_norm and self.max_grad_norm > 0:
            self._local.zero_()
            for u in range(self.w.num_units):
                s = self.shard_len[u]
                C.nvls_sumsq(self.gbuf.mc_addr(self.eng.grads[u], r * s), s, float(grad_scale), self._local)
            if self.local is not None:
                self.local.add_sumsq(self._local)
            C.symm_scalar_allreduce(h.id, 0, h.next_epoch(), self._local, self._sumsq)
            sq = self._sumsq
            self.last_sumsq = sq
        lr = self.current_lr()
        self.step_count += 1
        for u in range(self.w.num_units):
            s = self.shard_len[u]
            C.nvls_adamw(self.gbuf.mc_addr(self.eng.grads[u], r * s), self.pbuf.mc_addr(self.w.bufs[u], r * s),
                         self.w.bufs[u][r * s:(r + 1) * s], self.master.get(u), self.m[u], self.v[u], r * s,
                         float(grad_scale), lr, self.b1, self.b2, self.eps, self.wd, self.step_count, sq,
                         float(self.max_grad_norm or 0.0),
                         self.seed * 7919 + self.step_count * 104729 + u * 31 + r)
        if self.local is not None:
            self.local.step(sq, float(self.max_grad_norm or 0.0))
        h.barrier()                                   # every rank holds all new parameters
