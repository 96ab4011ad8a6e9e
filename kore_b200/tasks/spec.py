"""The operator-spec record shared by every task family (no side effects on import)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, Optional, Tuple

import torch

Inputs = Tuple[torch.Tensor, ...]


def _gen(seed: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def _randn(shape, seed, device, dtype, scale=1.0):
    g = _gen(seed, device)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * scale).to(dtype)


@dataclass
class OpSpec:
    name: str
    operation: str                                   # roofline op name
    entry: str                                       # function the candidate defines
    make_inputs: Callable[[Dict[str, int], int, str, torch.dtype], Inputs]
    reference: Callable[..., torch.Tensor]           # fp32 oracle
    baseline: Callable[..., torch.Tensor]            # vendor bar on B200
    seed_src: str
    shapes: Dict[str, object] = field(default_factory=dict)
    family: str = "core"
    dtype: str = "bf16"
    snr_threshold: Optional[float] = None
