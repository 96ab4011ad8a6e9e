"""tcgen05 GEMM vs cuBLAS (torch.matmul) on the Qwen3-14B layer shapes.

    python -m kore_b200.bench.gemm_bench [--tokens 8192]
"""
from __future__ import annotations

import argparse
import json

import torch

from kore_b200 import ops
from kore_b200.bench.timing import median_ms, time_cuda


def shapes(T: int):
    H, F, QKV = 5120, 17408, 7168
    return [
        ("qkv_fwd", T, QKV, H, False, True),
        ("o_fwd", T, H, 5120, False, True),
        ("gateup_fwd", T, 2 * F, H, False, True),
        ("down_fwd", T, H, F, False, True),
        ("down_dgrad", T, F, H, False, False),
        ("down_wgrad", H, F, T, True, False),
        ("gateup_wgrad", 2 * F, H, T, True, False),
    ]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--pair", type=int, default=-1, help="1: 2-CTA pair kernel, 0: one CTA per tile, -1: both")
    args = ap.parse_args(argv)
    C = ops.native()
    torch.manual_seed(0)
    res = []
    for name, M, N, K, a_t, b_t in shapes(args.tokens):
        A = torch.randn((K, M) if a_t else (M, K), device="cuda").bfloat16()
        B = torch.randn((N, K) if b_t else (K, N), device="cuda").bfloat16()
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        modes = [0, 1] if args.pair < 0 else [args.pair]
        per_mode = {}
        for mode in modes:
            old = C.gemm_set_pair_mode(mode)
            per_mode[mode] = median_ms(time_cuda(lambda: ops.mm(A, B, a_t=a_t, b_t=b_t, out=out), args.iters))
            C.gemm_set_pair_mode(old)
        ours = min(per_mode.values())
        At = A.t() if a_t else A
        Bt = B.t() if b_t else B
        cub = median_ms(time_cuda(lambda: torch.matmul(At, Bt, out=out), args.iters))
        fl = 2.0 * M * N * K
        ref = At.float() @ Bt.float()
        ops.mm(A, B, a_t=a_t, b_t=b_t, out=out)
        err = ((out.float() - ref).norm() / ref.norm()).item()
        r = {"op": name, "M": M, "N": N, "K": K, "ours_ms": round(ours, 4),
             "cublas_ms": round(cub, 4), "ours_tflops": round(fl / ours / 1e9, 1),
             "cublas_tflops": round(fl / cub / 1e9, 1), "rel_err": err,
             "tflops_by_mode": {("pair" if m else "single"): round(fl / t / 1e9, 1) for m, t in per_mode.items()}}
        print(json.dumps(r), flush=True)
        res.append(r)
    return res


if __name__ == "__main__":
    main()
