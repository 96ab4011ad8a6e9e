"""Speed-of-light (roofline) model for B200 (sm_100a).

T_min = max(FLOPs / peak_flops(dtype), bytes / HBM bandwidth), and the
attainment eta = T_min / T_measured used by the physics reward.

Peaks: the MEASURED copy bandwidth and cuBLAS bf16 throughput of this pool
(``MEASURED_PEAKS.json`` at the repo root, written per pod) when present;
otherwise the nominal B200 figures below; ``KORE_PEAK_*`` environment
variables override either. The per-operation FLOP/byte models follow the same
physics as the reference's table (kore/analysis/rooflines.py:153-282): GEMM
2MNK with operand+output traffic, norms/activations as streaming passes,
causal prefill attention at half the square, decode attention streaming K/V,
MoE as top-k expert GEMMs with all expert weights read once.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Optional, Tuple

REPO_ROOT = Path(__file__).resolve().parents[2]

# Nominal dense peaks (per GPU) and HBM3e bandwidth; sparse figures excluded.
NOMINAL = {
    "sm_100a": {
        "bf16_flops_per_s": 2.25e15, "fp16_flops_per_s": 2.25e15, "tf32_flops_per_s": 1.1e15,
        "fp8_flops_per_s": 4.5e15, "int8_flops_per_s": 4.5e15, "fp6_flops_per_s": 4.5e15,
        "fp4_flops_per_s": 9.0e15, "fp32_flops_per_s": 80e12,
        "hbm_bytes_per_s": 7.7e12, "l2_bytes": 126e6, "hbm_bytes": 180e9, "sms": 148,
        "nvlink_bytes_per_s": 900e9,
    },
}
ARCH_ALIASES = {"b200": "sm_100a", "sm_100": "sm_100a", "sm100": "sm_100a", "blackwell": "sm_100a"}


def detect_arch() -> str:
    a = os.environ.get("GPU_TARGET", "sm_100a").lower()
    return ARCH_ALIASES.get(a, a)


def measured_peaks(path: Optional[Path] = None) -> Optional[dict]:
    p = Path(path) if path else REPO_ROOT / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


def resolve_peaks(arch: Optional[str] = None, use_measured: bool = True) -> Dict[str, float]:
    """Peak table for ``arch``: nominal, replaced by measured values where the
    pool measured them (bf16 GEMM burst -> bf16/fp16, ratio-scaled fp8/fp4;
    copy bandwidth -> HBM), then KORE_PEAK_* overrides."""
    arch = ARCH_ALIASES.get((arch or detect_arch()).lower(), (arch or "sm_100a").lower())
    peaks = dict(NOMINAL.get(arch, NOMINAL["sm_100a"]))
    if use_measured:
        m = measured_peaks()
        if m:
            if m.get("bf16_tflops"):
                bf = float(m["bf16_tflops"]) * 1e12
                scale = bf / peaks["bf16_flops_per_s"]
                for k in ("bf16_flops_per_s", "fp16_flops_per_s", "tf32_flops_per_s", "fp8_flops_per_s",
                          "int8_flops_per_s", "fp6_flops_per_s", "fp4_flops_per_s"):
                    peaks[k] *= scale
            if m.get("hbm_gbs"):
                peaks["hbm_bytes_per_s"] = float(m["hbm_gbs"]) * 1e9
    for k in list(peaks):
        env = os.environ.get("KORE_PEAK_" + k.upper())
        if env:
            try:
                peaks[k] = float(env)
            except ValueError:
                pass
    return peaks


def dtype_bytes(dtype: str) -> float:
    d = (dtype or "").lower()
    if any(t in d for t in ("fp4", "e2m1")):
        return 0.5
    if any(t in d for t in ("fp6", "e2m3", "e3m2")):
        return 0.75
    if any(t in d for t in ("fp8", "float8", "int8")):
        return 1.0
    if any(t in d for t in ("fp32", "float32", "tf32")):
        return 4.0
    return 2.0


def peak_flops(peaks: Dict[str, float], dtype: str) -> float:
    d = (dtype or "").lower()
    for keys, name in ((("fp4", "e2m1"), "fp4_flops_per_s"), (("fp6", "e2m3", "e3m2"), "fp6_flops_per_s"),
                       (("fp8", "float8"), "fp8_flops_per_s"), (("int8",), "int8_flops_per_s"),
                       (("tf32",), "tf32_flops_per_s"), (("fp32", "float32"), "fp32_flops_per_s")):
        if any(k in d for k in keys):
            return peaks.get(name, peaks["bf16_flops_per_s"])
    return peaks["bf16_flops_per_s"]


def flops_bytes(operation: str, dims: Dict[str, int], dtype: str) -> Optional[Tuple[float, float]]:
    """(FLOPs, compulsory HBM bytes) of one call of ``operation`` at ``dims``."""
    op = (operation or "").lower()
    e = dtype_bytes(dtype)
    fp8 = "fp8" in (dtype or "").lower()

    def get(*names, default=None):
        for n in names:
            if n in dims:
                return dims[n]
        return default

    try:
        if any(t in op for t in ("batched_gemm", "grouped_gemm")) or op == "bmm":
            B = get("B", "batch", "num_batches", default=1)
            M, N, K = dims["M"], dims["N"], dims["K"]
            io = (M * K + K * N) * (1 if fp8 else e) + M * N * (2 if fp8 else e)
            return 2.0 * B * M * N * K, float(B * io)
        if "gemm" in op or "matmul" in op or op == "linear":
            if "K" not in dims and "N_out" in dims:
                # a fused pipeline's GEMM stage: the M x N input times an N_out x N weight
                M, N, K = dims["M"], dims["N_out"], dims["N"]
            else:
                M, N, K = dims["M"], dims["N"], dims["K"]
            io = (M * K + K * N) * (1 if fp8 else e) + M * N * (2 if fp8 else e)
            return 2.0 * M * N * K, float(io)
        if ("rmsnorm" in op and "fused" in op) or "fused_add" in op:
            M, N = dims["M"], dims["N"]
            return 5.0 * M * N, float((4 * M * N + N) * e)
        if "rmsnorm" in op:
            M, N = dims["M"], dims["N"]
            return 4.0 * M * N, float((2 * M * N + N) * e)
        if "layernorm" in op or "layer_norm" in op:
            M, N = dims["M"], dims["N"]
            return 6.0 * M * N, float((2 * M * N + 2 * N) * e)
        if ("silu" in op or "swiglu" in op) and "moe" not in op:
            M, N = dims["M"], dims["N"]
            return 4.0 * M * N, float(3 * M * N * e)
        if "gelu" in op or "relu" in op:
            M, N = dims["M"], dims["N"]
            return 8.0 * M * N, float(2 * M * N * e)
        if "topk" in op or "router" in op:
            M, E = dims["M"], dims["E"]
            k = get("topk", "k", default=max(1, E // 4))
            return 5.0 * M * E, float(M * E * e + M * k * (e + 4))
        if ("cross_entropy" in op or "logprob" in op or "log_softmax" in op):
            M, N = dims["M"], dims["N"]
            return 6.0 * M * N, float(2 * M * N * e)
        if op == "optimizer":
            N = dims["N"]                    # param + grad in the dtype, fp32 moments read and written
            return 12.0 * N, float(N * (3 * e + 16))
        if op == "newton_schulz":
            a, b = sorted((dims["M"], dims["N"]))
            return 5 * (4.0 * a * a * b + 2.0 * a ** 3), float(2 * a * b * e)
        if op == "loss_bwd":
            M, N = dims["M"], dims["N"]
            return 8.0 * M * N, float(2 * M * N * e)
        if op == "linear_attention":
            B, H, L, K = dims["B"], dims["H"], dims["L"], dims["K"]
            return 4.0 * B * H * L * K * K, float(5 * B * H * L * K * e)
        if "softmax" in op and "moe" not in op:
            M, N = dims["M"], get("N", "V")
            return 5.0 * M * N, float(2 * M * N * e)
        if "rope" in op:
            S, B, H, D = get("S", "T"), get("B", default=1), dims["H"], dims["D"]
            n = S * B * H * D
            return 6.0 * n, float(2 * n * e + S * D * e)
        if "quant" in op:
            M, N = dims["M"], dims["N"]
            return 2.0 * M * N, float(M * N * 3 + M * 4)
        if op == "moe_sum_combine":            # weighted sum of the top-k expert rows per token
            M, D, k = dims["M"], dims["D"], get("topk", "k", default=8)
            return 2.0 * M * k * D, float((M * k * D + M * D) * e + M * k * 8)
        if op in ("moe_permute", "moe_combine"):
            M, D, k = dims["M"], dims["D"], get("K", "topk", default=1)
            moved = M * k * D
            return float(moved if op == "moe_combine" else 0) * 2.0, float((moved + (M * D if op == "moe_combine" else M * D)) * e)
        if "moe" in op:
            M = dims["M"]
            E, k = get("E", "n_experts", default=8), get("topk", "k", default=2)
            D, I = get("D", "hidden", "d_model"), get("I", "inter", "d_ff")
            if D is None or I is None:
                return None
            return M * k * 6.0 * D * I, float((E * 3 * D * I + 2 * M * D) * e)
        if "attn" in op or "attention" in op:
            B, H, D = dims["B"], dims["H"], dims["D"]
            KV = get("KV", "kv_heads", default=H)
            if "decode" in op:
                Skv = get("Skv", "S_kv", "S", "seqlen")
                if Skv is None:
                    return None
                return 4.0 * B * H * Skv * D, float((2 * B * KV * Skv * D + 2 * B * H * D) * e)
            S = get("S", "seqlen")
            if S is None:
                return None
            return 2.0 * B * H * S * S * D, float((2 * B * H * S * D + 2 * B * KV * S * D) * e)
        size, seen = 1, False
        for v in dims.values():
            if isinstance(v, int) and v > 0:
                size *= v
                seen = True
        return (float(size), float(2 * size * e)) if seen else None
    except (KeyError, TypeError):
        return None


@dataclass
class Roofline:
    task_id: str
    operation: str
    dtype: str
    shape: str
    arch: str
    flops: float
    bytes: float
    arithmetic_intensity: float
    t_compute_ms: float
    t_mem_ms: float
    t_min_ms: float
    bound: str


def roofline(task_id: str, operation: str, dtype: str, shape_str: str, dims: Dict[str, int],
             peaks: Dict[str, float], arch: str) -> Optional[Roofline]:
    fb = flops_bytes(operation, dims, dtype)
    if fb is None or fb[1] <= 0:
        return None
    fl, by = fb
    tc = fl / peak_flops(peaks, dtype)
    tm = by / peaks["hbm_bytes_per_s"]
    return Roofline(task_id, operation, dtype, shape_str, arch, fl, by, fl / by, tc * 1e3, tm * 1e3,
                    max(tc, tm) * 1e3, "compute" if tc >= tm else "memory")


def shape_to_str(dims: Dict[str, int]) -> str:
    return ",".join(f"{k}={v}" for k, v in dims.items())


def eta(t_min_ms: float, measured_ms: float) -> Optional[float]:
    """Roofline attainment T_min / T_measured (capped at 1 is NOT applied here:
    values above 1 indicate a measurement problem)."""
    if not measured_ms or measured_ms <= 0 or not t_min_ms or t_min_ms <= 0:
        return None
    return t_min_ms / measured_ms


def fused_collective_roofline(flops: float, nvlink_bytes: float, peaks: Optional[dict] = None,
                              link_bytes_per_s: float = 770e9) -> float:
    """Target time (ms) of a fused compute+collective kernel: the slower of
    its math at the bf16 peak and its NVLink bytes at the per-direction link
    bandwidth (measured peer copy 770 GB/s on this pool)."""
    p = peaks or resolve_peaks()
    return max(flops / p["bf16_flops_per_s"], nvlink_bytes / link_bytes_per_s) * 1e3
