"""Device timing helpers: CUDA events on the launching stream, warm-up, and an
L2 flush (a write larger than the 126 MB L2) between timed iterations.

Reference parity: the reference's driver contract flushes L2 with a 256 MiB
buffer and times with CUDA events (kore/tasks/_genops.py:787-833)."""
from __future__ import annotations

import statistics
from typing import Callable

import torch

_FLUSH = {}


def l2_flush(device=None, nbytes: int = 512 << 20):
    dev = torch.device(device or "cuda")
    buf = _FLUSH.get(dev)
    if buf is None or buf.numel() < nbytes // 4:
        buf = torch.empty(nbytes // 4, dtype=torch.float32, device=dev)
        _FLUSH[dev] = buf
    buf.fill_(1.0)


def time_cuda(fn: Callable[[], object], iters: int = 10, warmup: int = 3,
              flush_l2: bool = True) -> list[float]:
    """Per-iteration device milliseconds of ``fn`` (events around each call)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        if flush_l2:
            l2_flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return out


def median_ms(xs: list[float]) -> float:
    return statistics.median(xs)
