"""Process-group plumbing: one process per GPU over NCCL (gloo on CPU).

Reads RANK / LOCAL_RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT from the
environment (torchrun / torch.distributed.run). Rendezvous defaults to
127.0.0.1.

Reference parity: the reference gets its process group from
``accelerate launch`` (scripts/launch_distributed.sh:91-112) and gathers
pickled objects with ``dist.all_gather_object`` (kore/policy/grpo.py:1518-1548).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Any, List, Optional

import torch
import torch.distributed as dist


@dataclass
class DistContext:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    backend: str = "none"
    group: Any = None

    @property
    def is_main(self) -> bool:
        return self.rank == 0

    @property
    def enabled(self) -> bool:
        return self.world > 1

    def barrier(self) -> None:
        if self.enabled:
            if self.backend == "nccl":
                dist.barrier(device_ids=[self.local_rank])
            else:
                dist.barrier()

    def all_reduce(self, t: torch.Tensor, op=None) -> torch.Tensor:
        if self.enabled:
            dist.all_reduce(t, op=op or dist.ReduceOp.SUM, group=self.group)
        return t

    def all_gather_object(self, obj) -> List[Any]:
        if not self.enabled:
            return [obj]
        out: List[Any] = [None] * self.world
        dist.all_gather_object(out, obj, group=self.group)
        return out

    def broadcast_object(self, obj, src: int = 0):
        if not self.enabled:
            return obj
        box = [obj]
        dist.broadcast_object_list(box, src=src, group=self.group)
        return box[0]

    def max_over_ranks(self, x: float) -> float:
        if not self.enabled:
            return x
        t = torch.tensor([x], dtype=torch.float64,
                         device=self.device if self.backend == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())


_CTX: Optional[DistContext] = None


def init_distributed(backend: Optional[str] = None, timeout_s: float = 1800.0) -> DistContext:
    """Initialise (once) from env vars; world 1 needs no process group."""
    global _CTX
    if _CTX is not None:
        return _CTX
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    cuda = torch.cuda.is_available()
    if backend is None:
        backend = "nccl" if cuda else "gloo"
    device = torch.device(f"cuda:{local}") if cuda and backend == "nccl" else torch.device("cpu")
    if cuda and backend == "nccl":
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        kw = dict(backend=backend, rank=rank, world_size=world,
                  timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(**kw)
    _CTX = DistContext(rank=rank, world=world, local_rank=local, device=device,
                       backend=backend if world > 1 else "none")
    return _CTX


def get_context() -> DistContext:
    return _CTX if _CTX is not None else DistContext(
        device=torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu"))


def shutdown() -> None:
    global _CTX
    if dist.is_initialized():
        dist.destroy_process_group()
    _CTX = None
