"""Parking device state in host memory between the phases of a training step.

A GRPO step on one GPU holds, at different times, the KV cache of the rollout,
the frozen reference model, and the optimizer moments; on a 14B model they do
not all fit in HBM at once. ``HostStash`` moves a set of device tensors to
(pinned) host buffers and back with stream-ordered asynchronous copies: the
device memory is released to the caching allocator as soon as the copies are
enqueued (a later allocation on the same stream is ordered after them), and
the host buffers are allocated once and reused every step.

Tensors are addressed as ``(container, key)`` slots (a dict entry or a list
index), so the owner keeps using its own attribute names; a parked slot holds
``None`` until it is restored.
"""
from __future__ import annotations

from typing import Any, Dict, List, Sequence, Tuple

import torch

Slot = Tuple[Any, Any]


class HostStash:
    def __init__(self, pin: bool = True):
        self.pin = pin
        self._host: Dict[int, torch.Tensor] = {}
        self.parked = False
        self.bytes = 0

    def park(self, slots: Sequence[Slot]) -> int:
        """Copy every slot's tensor to host and drop the device tensor."""
        if self.parked:
            return 0
        moved = 0
        for i, (c, k) in enumerate(slots):
            t = c[k]
            if t is None:
                continue
            h = self._host.get(i)
            if h is None or h.shape != t.shape or h.dtype != t.dtype:
                try:
                    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=self.pin and t.is_cuda)
                except RuntimeError:   # page-locking refused (host memory): pageable copies still work
                    self.pin = False
                    h = torch.empty(t.shape, dtype=t.dtype)
                self._host[i] = h
            h.copy_(t, non_blocking=True)
            moved += t.numel() * t.element_size()
            c[k] = None
        self.parked = True
        self.bytes = moved
        return moved

    def restore(self, slots: Sequence[Slot], device) -> int:
        """Bring the parked tensors back to ``device``."""
        if not self.parked:
            return 0
        moved = 0
        for i, (c, k) in enumerate(slots):
            h = self._host.get(i)
            if h is None or c[k] is not None:
                continue
            c[k] = h.to(device, non_blocking=True)
            moved += h.numel() * h.element_size()
        self.parked = False
        return moved


def optimizer_slots(opt) -> List[Slot]:
    """The per-unit state tensors of an AdamW-family optimizer: first and
    second moments and the fp32 master (when kept), including the local
    (expert) optimizer of an expert-parallel run."""
    out: List[Slot] = []
    for o in (opt, getattr(opt, "local", None)):
        if o is None:
            continue
        for name in ("m", "v", "master"):
            d = getattr(o, name, None)
            if isinstance(d, dict):
                out += [(d, k) for k in sorted(d)]
    return out


def weight_slots(weights) -> List[Slot]:
    out: List[Slot] = [(weights.bufs, i) for i in range(len(weights.bufs))]
    out += [(weights.expert_bufs, k) for k in sorted(weights.expert_bufs)]
    return out


def slots_bytes(slots: Sequence[Slot]) -> int:
    return sum(c[k].numel() * c[k].element_size() for c, k in slots if c[k] is not None)
