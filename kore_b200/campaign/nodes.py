"""Shared-node helpers: free-GPU picking (NVML, read-only queries) with retry,
and longest-processing-time-first partitioning of datagen work over workers.
Reference parity: scripts/run_grpo_resilient.sh:22-53, scripts/spur_partition.py.
"""
from __future__ import annotations

import heapq
import time
from typing import Callable, Dict, List, Optional, Sequence, Tuple


def gpu_usage(nvml=None) -> List[Tuple[int, int, int]]:
    """(index, used MiB, running compute processes) per GPU; read-only NVML queries."""
    if nvml is None:
        import pynvml as nvml
    nvml.nvmlInit()
    try:
        out = []
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            mem = nvml.nvmlDeviceGetMemoryInfo(h)
            procs = nvml.nvmlDeviceGetComputeRunningProcesses(h)
            out.append((i, int(mem.used) >> 20, len(procs)))
        return out
    finally:
        nvml.nvmlShutdown()


def pick_free_gpus(n: int, max_used_mib: int = 2048, retries: int = 10, wait_s: float = 30.0,
                   nvml=None, sleep: Callable[[float], None] = time.sleep) -> List[int]:
    for attempt in range(retries):
        free = [i for i, used, procs in gpu_usage(nvml) if procs == 0 and used <= max_used_mib]
        if len(free) >= n:
            return free[:n]
        if attempt + 1 < retries:
            sleep(wait_s)
    raise RuntimeError(f"fewer than {n} free GPUs after {retries} attempts")


def lpt_partition(costs: Dict[str, float], workers: int) -> List[List[str]]:
    """Longest-processing-time-first: assign each item (largest first) to the
    least-loaded worker; makespan within 4/3 of optimal."""
    heap = [(0.0, w) for w in range(workers)]
    parts: List[List[str]] = [[] for _ in range(workers)]
    for k, c in sorted(costs.items(), key=lambda kv: (-kv[1], kv[0])):
        load, w = heapq.heappop(heap)
        parts[w].append(k)
        heapq.heappush(heap, (load + c, w))
    return parts
