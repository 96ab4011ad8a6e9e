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


# ----------------------------------------------------------------------------- datagen arrays
def array_manifest(costs: Dict[str, float], shards: int, path: str) -> List[List[str]]:
    """Write an LPT partition of the work items as a JSON manifest (one list of
    task ids per array index) and return it; array task ``i`` reads entry ``i``."""
    import json
    parts = lpt_partition(costs, shards)
    with open(path, "w") as f:
        json.dump({"shards": parts, "costs": {k: float(v) for k, v in costs.items()}}, f, indent=1)
    return parts


def manifest_shard(path: str, index: int) -> List[str]:
    import json
    with open(path) as f:
        return list(json.load(f)["shards"][index])


def sbatch_array_script(manifest: str, kind: str, out_dir: str, *, shards: int, gpus_per_task: int = 1,
                        partition: Optional[str] = None, hours: int = 8, python: str = "python") -> str:
    """A SLURM array script: array task i runs ``kore datagen <kind>`` on the
    task ids of manifest entry i, writing ``<out_dir>/<kind>-shard<i>.jsonl``
    (resumable: a shard skips task ids it already holds)."""
    lines = ["#!/bin/bash", f"#SBATCH --job-name=kore-{kind}", f"#SBATCH --array=0-{shards - 1}",
             f"#SBATCH --gres=gpu:{gpus_per_task}", f"#SBATCH --time={hours}:00:00",
             f"#SBATCH --output={out_dir}/slurm-%A_%a.log"]
    if partition:
        lines.append(f"#SBATCH --partition={partition}")
    lines += ["set -euo pipefail",
              f"TASKS=$({python} -c \"from kore_b200.campaign.nodes import manifest_shard; "
              f"print(','.join(manifest_shard('{manifest}', $SLURM_ARRAY_TASK_ID)))\")",
              f"{python} -m kore_b200.cli datagen {kind} --tasks \"$TASKS\" "
              f"--out {out_dir}/{kind}-shard$SLURM_ARRAY_TASK_ID.jsonl"]
    return "\n".join(lines) + "\n"


def merge_shards(paths: Sequence[str], out: str, key: str = "task_id") -> int:
    """Concatenate JSONL shards, keeping the first record per (key, kernel hash)."""
    import hashlib
    import json
    seen, n = set(), 0
    with open(out, "w") as fo:
        for p in paths:
            try:
                fh = open(p)
            except OSError:
                continue
            with fh:
                for line in fh:
                    if not line.strip():
                        continue
                    try:
                        r = json.loads(line)
                    except json.JSONDecodeError:
                        continue
                    h = (r.get(key), hashlib.sha1(str(r.get("kernel", r.get("completion", ""))).encode()).hexdigest())
                    if h in seen:
                        continue
                    seen.add(h)
                    fo.write(json.dumps(r) + "\n")
                    n += 1
    return n
