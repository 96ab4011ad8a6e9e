"""Symmetric peer-memory heap (CUDA IPC over NVLink / NVSwitch).

Every rank allocates one heap of the same size; IPC handles are exchanged
over the process group and each rank maps every peer's heap. ``alloc``
carves tensors at identical offsets on all ranks (bump allocator, 256-byte
aligned), so a kernel reaches peer p's copy of a tensor at
``peer_base[p] + offset``. The first 4 KB are the signal pad of the
epoch-tagged device barriers. Lifetime: the heap lives until process exit.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from ..ops import native
from .dist import DistContext

SIGNAL_BYTES = 4096


class SymmetricHeap:
    def __init__(self, ctx: DistContext, nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes) + SIGNAL_BYTES
        C = native()
        self.id = C.symm_heap_create(self.nbytes, ctx.rank, ctx.world)
        if ctx.world > 1:
            h = C.symm_heap_handle(self.id)
            hs = ctx.all_gather_object(h.tolist())
            C.symm_heap_open(self.id, torch.tensor(hs, dtype=torch.uint8))
        self.offset = SIGNAL_BYTES
        self.epoch = 0
        self.tensors: Dict[int, Tuple[int, torch.Tensor]] = {}

    def alloc(self, numel: int, dtype=torch.bfloat16) -> Tuple[int, torch.Tensor]:
        esz = torch.empty((), dtype=dtype).element_size()
        off = (self.offset + 255) // 256 * 256
        end = off + int(numel) * esz
        if end > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted ({end} > {self.nbytes} bytes)")
        t = native().symm_heap_tensor(self.id, off, [int(numel)], dtype)
        self.offset = end
        self.tensors[t.data_ptr()] = (off, t)
        return off, t

    def offset_of(self, t: torch.Tensor) -> int:
        base_off, base = self.tensors[t.untyped_storage().data_ptr()]
        return base_off + (t.data_ptr() - base.data_ptr())

    def barrier(self) -> None:
        """Device-side barrier across all ranks on the current stream."""
        if self.ctx.world > 1:
            self.epoch += 1
            native().symm_barrier(self.id, 0, self.epoch)

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch
