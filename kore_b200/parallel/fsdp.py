"""Full sharding (ZeRO-3 / FSDP FULL_SHARD) of the decoder layers.

Each rank keeps only its 1/world shard of every decoder-layer unit (bf16
parameters, gradient accumulator, AdamW moments, optional fp32 master).
Full layer parameters exist only transiently, in a ring of two gathered
buffers; layer gradients likewise in a ring of two full buffers:

  forward   unit u: wait gather(u); issue gather(u+1) on the comm stream
  backward  unit u: wait gather(u); issue gather(u-1); recompute + backward
            into a gradient ring slot; then reduce-scatter that slot into
            the rank's gradient shard on the comm stream, overlapped with the
            backward of u-1.

The embedding and head units (a vocabulary-sized matrix each) stay resident
and use the ZeRO-2 step (reduce-scatter, sharded AdamW, all-gather).

With ``peer_gather`` (the trainer's ``comm="fused"`` at ZeRO-3) the layer
shards live in a symmetric peer-memory heap and each gather is one
``cudaMemcpyAsync`` per rank on the comm stream: NVLink peer reads executed by
the copy engines, so the gathers take no SM time from the GEMMs they overlap
and need no NCCL kernel. Device barriers before and after the optimizer step
order every rank's shard update against the other ranks' reads.

Why gather into HBM rather than fusing the gather into the consuming GEMM:
a weight tile is read by every M tile of the GEMM (T/128 times per pass,
three passes per layer with recompute), so streaming it from a peer inside
the GEMM would move T/128 times the layer's bytes over NVLink. One gather
per use moves it once, and with HBM at 180 GB the two-slot ring costs
2 x 0.8 GB (a 14B layer), overlapped with the previous unit's compute.

Reference parity: FSDP FULL_SHARD with transformer-layer auto-wrap,
backward_prefetch=BACKWARD_PRE, forward_prefetch, limit_all_gathers
(kore/policy/configs.py:580-651; configs/accelerate_fsdp.yaml:50).
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .. import ops
from .dist import DistContext
from .zero import ShardedAdamW


class FullShard:
    """Parameter / gradient provider hooked into :class:`Qwen3Engine`."""

    def __init__(self, weights, engine, ctx: DistContext, peer_gather: bool = False):
        self.w, self.eng, self.ctx = weights, engine, ctx
        W, r = ctx.world, ctx.rank
        self.units = list(range(1, weights.num_units - 1))
        kinds = {weights.layouts[u].kind for u in self.units}
        n = {weights.padded_numel(u) for u in self.units}
        if len(kinds) != 1 or len(n) != 1:
            raise ValueError("full sharding needs identical decoder-layer layouts")
        self.n = n.pop()
        assert self.n % W == 0
        self.s = self.n // W
        dev = weights.device
        self.cuda = dev.type == "cuda" and ctx.backend == "nccl"
        self.pshard: Dict[int, torch.Tensor] = {}
        self.gshard: Dict[int, torch.Tensor] = {}
        self.heap, self.poff = None, {}
        if peer_gather and self.cuda:
            from .symmetric import SymmetricHeap
            esz = torch.empty((), dtype=weights.dtype).element_size()
            self.heap = SymmetricHeap(ctx, len(self.units) * (self.s * esz + 256))
        for u in self.units:
            src = weights.bufs[u][r * self.s:(r + 1) * self.s]
            if self.heap is not None:
                self.poff[u], self.pshard[u] = self.heap.alloc(self.s, weights.dtype)
                self.pshard[u].copy_(src)
            else:
                self.pshard[u] = src.clone()
            self.gshard[u] = torch.zeros(self.s, dtype=engine.grad_dtype, device=dev)
            weights.bufs[u] = None                     # drop the full copy
            engine.grads[u] = None
        if dev.type == "cuda":
            torch.cuda.empty_cache()
        self.pslot = [torch.empty(self.n, dtype=weights.dtype, device=dev) for _ in range(2)]
        self.gslot = [torch.zeros(self.n, dtype=engine.grad_dtype, device=dev) for _ in range(2)]
        self.rs_tmp = [torch.empty(self.s, dtype=engine.grad_dtype, device=dev) for _ in range(2)]
        self.owner = [-1, -1]
        self.comm = torch.cuda.Stream(device=dev) if self.cuda else None
        self.gather_ev = [None, None]
        self.rs_ev = [None, None]
        self.acc_started = {u: False for u in self.units}

    # ------------------------------------------------------------ gather
    def _gather(self, u: int) -> None:
        k = u % 2
        if self.owner[k] == u:
            return
        self.owner[k] = u
        if not self.cuda:
            parts = [torch.empty_like(self.pshard[u]) for _ in range(self.ctx.world)]
            dist.all_gather(parts, self.pshard[u], group=self.ctx.group)
            self.pslot[k].copy_(torch.cat(parts))
            return
        free = torch.cuda.Event()
        free.record()                                  # compute that last read this slot is enqueued
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(free)
            if self.heap is not None:        # copy-engine peer reads: no SMs, no NCCL kernel
                ops.native().symm_gather_ce(self.heap.id, self.poff[u], self.s * self.pshard[u].element_size(),
                                            self.pslot[k])
            else:
                dist.all_gather_into_tensor(self.pslot[k], self.pshard[u], group=self.ctx.group)
            ev = torch.cuda.Event()
            ev.record()
        self.gather_ev[k] = ev

    def sync_shards(self) -> None:
        """Device barrier over the ranks (peer-gather mode): orders every
        rank's shard update against the other ranks' next reads of it."""
        if self.heap is not None:
            self.heap.barrier()

    def acquire(self, u: int, nxt: Optional[int] = None) -> None:
        if u not in self.pshard:
            return
        self._gather(u)
        k = u % 2
        if self.cuda and self.gather_ev[k] is not None:
            torch.cuda.current_stream().wait_event(self.gather_ev[k])
        self.w.bufs[u] = self.pslot[k]
        if nxt is not None and nxt in self.pshard:
            self._gather(nxt)

    def release(self, u: int) -> None:
        if u in self.pshard:
            self.w.bufs[u] = None

    # ------------------------------------------------------------ gradients
    def begin_bwd(self, u: int) -> None:
        if u not in self.pshard:
            return
        k = u % 2
        if self.cuda and self.rs_ev[k] is not None:
            torch.cuda.current_stream().wait_event(self.rs_ev[k])   # slot's previous reduce-scatter done
        self.eng.grads[u] = self.gslot[k]
        self.eng._fresh[u] = True                      # overwrite: the slot held another unit

    def end_bwd(self, u: int) -> None:
        if u not in self.pshard:
            return
        k = u % 2
        g, acc, dst, tmp = self.gslot[k], self.acc_started[u], self.gshard[u], self.rs_tmp[k]
        self.eng.grads[u] = None
        self.acc_started[u] = True
        if not self.cuda:
            dist.all_reduce(g, group=self.ctx.group)
            part = g[self.ctx.rank * self.s:(self.ctx.rank + 1) * self.s]
            dst.add_(part) if acc else dst.copy_(part)
            return
        done = torch.cuda.Event()
        done.record()
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(done)
            if acc:
                dist.reduce_scatter_tensor(tmp, g, op=dist.ReduceOp.SUM, group=self.ctx.group)
                dst.add_(tmp)
            else:
                dist.reduce_scatter_tensor(dst, g, op=dist.ReduceOp.SUM, group=self.ctx.group)
            ev = torch.cuda.Event()
            ev.record()
        self.rs_ev[k] = ev

    def finish(self) -> None:
        """Join the comm stream (call before reading gradient shards)."""
        if self.cuda:
            torch.cuda.current_stream().wait_stream(self.comm)

    def zero_grad(self) -> None:
        for u in self.units:
            self.acc_started[u] = False
            self.gshard[u].zero_()

    # ------------------------------------------------------------ checkpoints
    @torch.no_grad()
    def full_unit(self, u: int) -> torch.Tensor:
        """A freshly gathered copy of unit u (for saving)."""
        if u not in self.pshard:
            return self.w.bufs[u]
        out = torch.empty(self.n, dtype=self.w.dtype, device=self.w.device)
        if self.ctx.backend == "nccl":
            dist.all_gather_into_tensor(out, self.pshard[u], group=self.ctx.group)
        else:
            parts = [torch.empty_like(self.pshard[u]) for _ in range(self.ctx.world)]
            dist.all_gather(parts, self.pshard[u], group=self.ctx.group)
            out.copy_(torch.cat(parts))
        return out


class FullShardAdamW(ShardedAdamW):
    """AdamW over ZeRO-3 layer shards (gradients already reduce-scattered
    during the backward; no all-gather after the update: the next forward
    gathers) plus ZeRO-2 for the resident embedding / head units."""

    def __init__(self, weights, engine, ctx, fs: FullShard, **kw):
        self.fs = fs
        # the parent sizes state from weights.bufs: present full buffers of the sharded units
        saved = {u: weights.bufs[u] for u in fs.units}
        for u in fs.units:
            weights.bufs[u] = fs.pslot[0]
        super().__init__(weights, engine, ctx, **kw)
        for u in fs.units:
            weights.bufs[u] = saved[u]
            self.gshard.pop(u, None)
            if u in self.master:
                self.master[u] = fs.pshard[u].float()

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, scattered: bool = False) -> None:
        fs, r = self.fs, self.ctx.rank
        fs.finish()
        fs.sync_shards()                               # every rank's last gather of this step is done
        resident = [u for u in range(self.w.num_units) if u not in fs.pshard]
        for u in resident:
            self.reduce_scatter_unit(u)
        gsh = lambda u: fs.gshard[u] if u in fs.pshard else self.gshard[u]
        sq = None
        if self.max_grad_norm and self.max_grad_norm > 0:
            self._sumsq.zero_()
            for u in range(self.w.num_units):
                ops.sumsq(gsh(u), self._sumsq)
            if self.local is not None:
                self.local.add_sumsq(self._sumsq)
            self.ctx.all_reduce(self._sumsq)
            sq = self._sumsq
            self.last_sumsq = sq
        if self.local is not None:
            self.local.step(sq, float(self.max_grad_norm or 0.0))
        lr = self.current_lr()
        self.step_count += 1
        for u in range(self.w.num_units):
            s = self.shard_len[u]
            p = fs.pshard[u] if u in fs.pshard else self.w.bufs[u][r * s:(r + 1) * s]
            kw = dict(lr=lr, b1=self.b1, b2=self.b2, eps=self.eps, wd=self.wd, step=self.step_count,
                      grad_scale=grad_scale, sumsq_buf=sq, max_norm=self.max_grad_norm)
            ops.adamw_step(p, gsh(u), self.m[u], self.v[u], master=self.master.get(u),
                           seed=self.seed * 7919 + self.step_count * 104729 + u * 31 + r, **kw)
            if u not in fs.pshard:
                self.all_gather_unit(u)
        fs.owner = [-1, -1]                            # gathered copies are stale now
        fs.sync_shards()                               # shards updated everywhere before the next gathers
        fs.zero_grad()
