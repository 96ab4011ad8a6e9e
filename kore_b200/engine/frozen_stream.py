"""Frozen models whose decoder layers do not stay in HBM.

The frozen reference model of DPO / GRPO is only read, one layer at a time,
during the reference forward. ``FrozenLayerStream`` keeps its decoder layers
elsewhere and brings each into a two-slot device ring just before the engine
needs it, overlapped with the previous layer's compute on a copy stream:

* ``source="host"``: layers live in pinned host memory and stream over PCIe
  (one GPU: the 14B policy with its optimizer state leaves no room for a
  second resident copy of the weights);
* ``source="shard"``: every rank keeps 1/world of each layer and the layer is
  all-gathered over NVLink (the reference "sharded alongside the policy").

Embedding and head units stay resident. The hook has the interface the engine
calls around each layer (``acquire(u, next)``); see
:class:`kore_b200.parallel.fsdp.FullShard` for the training-side counterpart.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch


class FrozenLayerStream:
    def __init__(self, weights, *, source: str = "host", ctx=None, layers_from=None):
        """``weights``: the frozen model (its decoder-layer buffers are taken over).
        ``layers_from``: another model whose current decoder layers are copied
        instead (e.g. the policy at step 0), leaving it untouched, so no second
        full device copy is ever made."""
        if source not in ("host", "shard"):
            raise ValueError("source must be host|shard")
        self.w, self.source, self.ctx = weights, source, ctx
        dev = weights.device
        self.cuda = dev.type == "cuda"
        self.units = list(range(1, weights.num_units - 1))
        self.n = max(weights.padded_numel(u) for u in self.units)
        self.store: Dict[int, torch.Tensor] = {}
        if source == "shard":
            W, r = ctx.world, ctx.rank
            assert self.n % W == 0, "pad the layer units to a multiple of the world size"
            self.s = self.n // W
        src = layers_from if layers_from is not None else weights
        for u in self.units:
            b = src.bufs[u]
            if source == "host":
                h = torch.empty(b.numel(), dtype=b.dtype, pin_memory=self.cuda)
                h.copy_(b)
                self.store[u] = h
            else:
                full = torch.zeros(self.n, dtype=b.dtype, device=dev)
                full[: b.numel()].copy_(b)
                self.store[u] = full[r * self.s:(r + 1) * self.s].clone()
                del full
            if layers_from is None:
                weights.bufs[u] = None
        if self.cuda:
            torch.cuda.empty_cache()
        self.slot = [torch.empty(self.n, dtype=weights.dtype, device=dev) for _ in range(2)]
        self.owner = [-1, -1]
        self.ev: list = [None, None]
        self.copy_stream = torch.cuda.Stream(device=dev) if self.cuda else None
        self.bytes_moved = 0

    def free_ring(self) -> None:
        """Release the two device slots (the layers stay in their store); the
        model's views into them are dropped too."""
        for u in self.store:
            self.w.bufs[u] = None
        self.slot = [None, None]
        self.owner = [-1, -1]
        self.ev = [None, None]

    def _fetch(self, u: int) -> None:
        k = u % 2
        if self.slot[k] is None:
            self.slot[k] = torch.empty(self.n, dtype=self.w.dtype, device=self.w.device)
        if self.owner[k] == u:
            return
        self.owner[k] = u
        numel = self.w.padded_numel(u)
        if not self.cuda:
            self._copy_into(k, u, numel)
            return
        free = torch.cuda.Event()
        free.record()                                    # compute that last read this slot is enqueued
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(free)
            self._copy_into(k, u, numel)
            ev = torch.cuda.Event()
            ev.record()
        self.ev[k] = ev

    def _copy_into(self, k: int, u: int, numel: int) -> None:
        if self.source == "host":
            self.slot[k][:numel].copy_(self.store[u], non_blocking=True)
            self.bytes_moved += self.store[u].numel() * self.store[u].element_size()
        else:
            import torch.distributed as dist
            if self.ctx.world > 1:
                dist.all_gather_into_tensor(self.slot[k], self.store[u], group=self.ctx.group)
            else:
                self.slot[k].copy_(self.store[u])

    def acquire(self, u: int, nxt: Optional[int] = None) -> None:
        if u not in self.store:
            return
        self._fetch(u)
        k = u % 2
        if self.cuda and self.ev[k] is not None:
            torch.cuda.current_stream().wait_event(self.ev[k])
        self.w.bufs[u] = self.slot[k][: self.w.padded_numel(u)]
        if nxt is not None and nxt in self.store:
            self._fetch(nxt)

    def release(self, u: int) -> None:
        if u in self.store:
            self.w.bufs[u] = None

    # the engine calls these around backward; a frozen model has none
    def begin_bwd(self, u: int) -> None:
        pass

    def end_bwd(self, u: int) -> None:
        pass

    def zero_grad(self) -> None:
        pass
