"""Feature vectors for the value model: the candidate's schedule plus the
task's context.

A candidate is either a Triton kernel or a CUDA C++ kernel (inline
extension); the schedule features read both kinds of source:

* Triton: tile sizes (BLOCK_M/N/K, BM/BN/BK, BLOCK), num_warps, num_stages,
  GROUP_SIZE_M, ``tl.dot``, fp32 accumulators, masks, K loops, exp2,
  contiguity hints, atomics;
* CUDA: the tensor-core tier it uses (tcgen05 > mma.sync > wmma > none), TMA
  (``cp.async.bulk``), cp.async, thread-block clusters, ``__launch_bounds__``
  threads, constexpr tile sizes, static shared memory bytes, 16-byte vector
  accesses, warp shuffles, atomics, unrolled loops, barriers;
* shared: loop count and source length.

Task context: dtype one-hot, operation-class one-hot, log2 of the primary
shape's sizes (largest four), log arithmetic intensity and a memory-bound flag
from the roofline model. All numbers are log-scaled or 0/1 so a linear head
works without further engineering. ``FEATURE_NAMES`` documents every slot.

Reference parity: the reference's featurizer (kore/value/features.py:62-400:
dtype / operation / bottleneck one-hots, dims, schedule vector from the
Triton source), extended to CUDA sources and sm_100a mechanisms.
"""
from __future__ import annotations

import math
import re
from typing import Dict, Iterable, List, Optional, Sequence

import numpy as np

DTYPES = ("bf16", "fp16", "fp32", "fp8", "int8", "fp4")
OP_CLASSES = ("gemm", "attention", "norm", "elementwise", "reduce", "moe", "conv", "ssm", "quant", "sample",
              "train", "other")
TC_TIERS = ("tcgen05", "mma_sync", "wmma", "none")
_TRITON_KNOBS = (("BLOCK_M", "BM"), ("BLOCK_N", "BN"), ("BLOCK_K", "BK"), ("BLOCK", "BLOCK_SIZE"),
                 ("num_warps",), ("num_stages",), ("GROUP_SIZE_M", "GROUP_M"))


def _log2p(x: Optional[float]) -> float:
    return math.log2(1.0 + max(0.0, float(x))) if x else 0.0


def _first_int(src: str, names: Sequence[str]) -> Optional[int]:
    for n in names:
        m = re.search(rf"\b{n}\s*(?::\s*tl\.constexpr\s*)?[=:]\s*(\d+)", src)
        if m:
            return int(m.group(1))
    return None


def norm_dtype(dtype: str) -> str:
    d = (dtype or "").lower()
    for k, al in (("fp8", ("fp8", "e4m3", "e5m2")), ("fp4", ("fp4", "mxfp4", "nvfp4")), ("int8", ("int8", "i8")),
                  ("bf16", ("bf16", "bfloat16")), ("fp16", ("fp16", "float16", "half")),
                  ("fp32", ("fp32", "float32", "float"))):
        if any(a in d for a in al):
            return k
    return "bf16"


def op_class(operation: str) -> str:
    o = (operation or "").lower()
    table = (("moe", ("moe", "expert", "router", "topk_router")), ("attention", ("attn", "attention", "mla")),
             ("quant", ("quant", "fp8", "int8", "int4", "mxfp", "nf4")), ("conv", ("conv", "pool")),
             ("ssm", ("scan", "ssm", "linear_attention", "recurrence")),
             ("train", ("adam", "lion", "sgd", "backward", "_bwd", "grad", "cross_entropy")),
             ("sample", ("sample", "top_p", "top_k", "min_p", "temperature")),
             ("norm", ("norm",)), ("gemm", ("gemm", "matmul", "linear", "bmm")),
             ("reduce", ("reduce", "softmax", "sum", "max", "mean", "argmax", "logsumexp")))
    for k, keys in table:
        if any(x in o for x in keys):
            return k
    return "elementwise" if o else "other"


def tensor_core_tier(src: str) -> str:
    if "tcgen05" in src:
        return "tcgen05"
    if "mma.sync" in src or "mma_sync(" in src and "wmma" not in src:
        return "mma_sync"
    if "wmma::" in src or "nvcuda::wmma" in src:
        return "wmma"
    return "none"


def _smem_bytes(src: str) -> int:
    """Static shared-memory bytes declared as fixed-size arrays."""
    size = {"float": 4, "int": 4, "half": 2, "__half": 2, "__nv_bfloat16": 2, "double": 8, "uint8_t": 1,
            "char": 1, "float4": 16, "uint4": 16, "int4": 16, "uint32_t": 4, "uint64_t": 8}
    tot = 0
    for m in re.finditer(r"__shared__\s+(?:__align__\(\d+\)\s+)?(\w+)\s+\w+((?:\[\d+\])+)", src):
        n = 1
        for d in re.findall(r"\[(\d+)\]", m.group(2)):
            n *= int(d)
        tot += n * size.get(m.group(1), 4)
    return tot


def schedule_features(src: str) -> Dict[str, float]:
    s = src or ""
    f: Dict[str, float] = {}
    for names in _TRITON_KNOBS:
        v = _first_int(s, names)
        f["log2_" + names[0].lower()] = math.log2(v) if v else 0.0
    f["tl_dot"] = float("tl.dot(" in s)
    f["fp32_acc"] = float(bool(re.search(r"tl\.zeros\([^\n]*float32", s) or re.search(r"float\s+acc", s)))
    f["masked"] = float("mask=" in s or "if (" in s and "< n" in s.lower())
    f["k_loop"] = float(bool(re.search(r"for \w+ in (tl\.)?(static_)?range\(", s)))
    f["exp2"] = float("exp2" in s)
    f["contiguity_hints"] = float("multiple_of" in s or "max_contiguous" in s)
    tier = tensor_core_tier(s)
    for t in TC_TIERS:
        f["tc_" + t] = float(tier == t)
    f["tma"] = float("cp.async.bulk" in s or "CUtensorMap" in s or "tma_load" in s)
    f["cp_async"] = float("cp.async" in s and "cp.async.bulk" not in s)
    f["cluster"] = float("__cluster_dims__" in s or "cudaLaunchKernelEx" in s or "cluster_dims" in s)
    lb = re.search(r"__launch_bounds__\(\s*(\d+)", s)
    f["log2_threads"] = math.log2(int(lb.group(1))) if lb else 0.0
    tiles = [int(x) for x in re.findall(r"constexpr\s+int\s+(?:BM|BN|BK|TILE\w*|kBlock\w*)\s*=\s*(\d+)", s)]
    f["log2_max_tile"] = math.log2(max(tiles)) if tiles else 0.0
    f["log2_smem"] = _log2p(_smem_bytes(s) + (65536 if "extern __shared__" in s else 0))
    f["vec16"] = float(bool(re.search(r"\b(float4|uint4|int4)\b", s)))
    f["shuffles"] = _log2p(len(re.findall(r"__shfl_\w+sync", s)))
    f["atomics"] = float("atomicAdd" in s or "tl.atomic" in s or "red.global" in s)
    f["unroll"] = _log2p(s.count("#pragma unroll"))
    f["barriers"] = _log2p(s.count("__syncthreads") + s.count("bar.sync") + s.count("mbarrier"))
    f["loops"] = _log2p(len(re.findall(r"\bfor\s*\(|\bfor \w+ in ", s)))
    f["log_len"] = math.log1p(len(s))
    return f


def task_features(meta: Optional[dict]) -> Dict[str, float]:
    """``meta``: {"dtype", "operation", "dims": {...}, "intensity", "bound"}
    (any may be missing)."""
    meta = meta or {}
    f: Dict[str, float] = {}
    d = norm_dtype(meta.get("dtype", ""))
    for k in DTYPES:
        f["dtype_" + k] = float(d == k)
    oc = op_class(meta.get("operation", ""))
    for k in OP_CLASSES:
        f["op_" + k] = float(oc == k)
    sizes = sorted((float(v) for v in (meta.get("dims") or {}).values() if isinstance(v, (int, float)) and v > 0),
                   reverse=True)[:4]
    sizes += [0.0] * (4 - len(sizes))
    for i, v in enumerate(sizes):
        f[f"log2_dim{i}"] = _log2p(v)
    f["log_intensity"] = math.log1p(max(0.0, float(meta.get("intensity") or 0.0)))
    f["memory_bound"] = float(meta.get("bound") == "memory")
    return f


def _names() -> List[str]:
    return list(schedule_features("").keys()) + list(task_features({}).keys()) + ["bias"]


FEATURE_NAMES: List[str] = _names()


def featurize(src: str, meta: Optional[dict] = None) -> np.ndarray:
    f = schedule_features(src)
    f.update(task_features(meta))
    f["bias"] = 1.0
    return np.asarray([f[n] for n in FEATURE_NAMES], dtype=np.float64)


def featurize_many(sources: Iterable[str], meta: Optional[dict] = None) -> np.ndarray:
    rows = [featurize(s, meta) for s in sources]
    return np.stack(rows) if rows else np.zeros((0, len(FEATURE_NAMES)))


def task_meta(task) -> dict:
    """The context ``task_features`` reads, from a task of the registry."""
    if task is None:
        return {}
    meta = {"dtype": getattr(task, "dtype", ""), "operation": getattr(task, "operation", "")}
    try:
        sh = task.shape("primary") or task.shapes[0]
        meta["dims"] = dict(sh.dims)
        from ..analysis.rooflines import flops_bytes
        fb = flops_bytes(task.operation, sh.dims, task.dtype)
        if fb and fb[1]:
            meta["intensity"] = fb[0] / fb[1]
            meta["bound"] = "compute" if meta["intensity"] > 300 else "memory"
    except Exception:  # noqa: BLE001 - context is optional
        pass
    return meta


def meta_from_record(task_id: str, operation: Optional[str] = None, shape: Optional[str] = None) -> dict:
    """Context for a stored record: the registry task when it is known, else
    what the record carries."""
    try:
        from ..tasks.registry import get_task
        return task_meta(get_task(task_id))
    except Exception:  # noqa: BLE001
        m = re.search(r"_(bf16|fp16|fp32|fp8|int8|fp4)\b", task_id or "")
        return {"operation": operation or task_id, "dtype": m.group(1) if m else ""}


def synthesize_groups(n_groups: int, group_size: int = 6, seed: int = 0) -> List[List[dict]]:
    """Synthetic ranked groups with a known ground truth, for cold start and
    tests: Triton GEMM candidates whose speedup rises with tensor-core use,
    64-multiple tiles, 4-8 warps and 2-4 stages (plus noise); tiny tiles
    sometimes fail to compile and unmasked edges sometimes fail correctness.
    Rows: {"source", "compiled", "correct", "speedup", "meta"}."""
    rng = np.random.default_rng(seed)
    groups = []
    for _ in range(n_groups):
        M = int(rng.choice([1024, 2048, 4096, 8192]))
        meta = {"dtype": str(rng.choice(["bf16", "fp16"])), "operation": "gemm",
                "dims": {"M": M, "N": M, "K": M}, "intensity": M / 3.0, "bound": "compute"}
        rows = []
        for _ in range(group_size):
            bm, bn, bk = (int(rng.choice([16, 32, 64, 128, 256])) for _ in range(3))
            warps, stages = int(rng.choice([1, 2, 4, 8, 16])), int(rng.choice([1, 2, 3, 4, 6]))
            dot, masked = bool(rng.random() < 0.7), bool(rng.random() < 0.8)
            src = (f"BLOCK_M = {bm}\nBLOCK_N = {bn}\nBLOCK_K = {bk}\nnum_warps = {warps}\nnum_stages = {stages}\n"
                   + ("acc = tl.zeros((BLOCK_M, BLOCK_N), dtype=tl.float32)\n" if dot else "")
                   + "for k in range(0, K, BLOCK_K):\n"
                   + ("    acc += tl.dot(a, b)\n" if dot else "    acc += tl.sum(a[:, :, None] * b[None], 1)\n")
                   + ("    a = tl.load(pa, mask=m)\n" if masked else "    a = tl.load(pa)\n"))
            score = (1.2 * dot + 0.3 * (bm % 64 == 0) + 0.3 * (bn % 64 == 0) + 0.2 * (warps in (4, 8))
                     + 0.2 * (2 <= stages <= 4) - 0.4 * (bm * bn > 128 * 256))
            compiled = not (bm * bn * bk > 256 * 256 * 64) and rng.random() > 0.05
            correct = compiled and (masked or rng.random() < 0.5)
            speed = float(np.exp(score - 1.0 + 0.15 * rng.standard_normal())) if correct else None
            rows.append({"source": src, "compiled": compiled, "correct": correct, "speedup": speed,
                         "meta": meta})
        groups.append(rows)
    return groups
