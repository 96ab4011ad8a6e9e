"""MoE gate/up grouped GEMM on one GPU, Qwen3-Coder-30B-A3B shape.

    python -m kore_b200.bench.moe_bench [--tokens 8192] [--iters 10]

Times, with CUDA events after warm-up and L2 flushed between iterations:
(1) the device routing plan's row gather (tokens into the padded
expert-major order) followed by the grouped tcgen05 GEMM over the device
tile table, and (2) the grouped GEMM that stages its own receive rows in its
prologue from a token buffer addressed by an index (the expert-parallel pull
dispatch, with this GPU as the only peer). The difference is the cost of
staging inside the GEMM launch against a separate gather pass; on several
GPUs the remote rows come over NVLink instead.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops
from ..ops import moe as M
from .timing import median_ms, time_cuda


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=768)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    from ..parallel.dist import DistContext
    from ..parallel.symmetric import SymmetricHeap
    C = ops.native()
    T, E, k, H, N = a.tokens, a.experts, a.topk, a.hidden, 2 * a.inter
    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    idx = torch.randn(T, E, device=dev, generator=g).topk(k, -1).indices.int().contiguous()
    w = (torch.randn(E, N, H, device=dev, generator=g) * 0.02).bfloat16()
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    p = M.plan(idx, E)
    cap = (p.rows + 63) // 64 * 64
    heap = SymmetricHeap(DistContext(device=dev), T * H * 2 + (1 << 16))
    o_tok, tok = heap.alloc(T * H)
    tok.view(T, H).copy_(x)
    peers = C.symm_peer_addrs(heap.id, o_tok)
    index = torch.full((cap,), -1, dtype=torch.int32, device=dev)
    index[: p.rows] = p.src_row
    flags = torch.zeros(cap // 64, dtype=torch.int32, device=dev)
    stage = torch.empty(cap, H, dtype=torch.bfloat16, device=dev)
    out = torch.empty(cap, N, dtype=torch.bfloat16, device=dev)
    xg = torch.empty(p.rows, H, dtype=torch.bfloat16, device=dev)
    out2 = torch.empty(p.rows, N, dtype=torch.bfloat16, device=dev)
    epoch = [0]

    def gathered():
        C.moe_gather_rows(x, p.src_row, xg)
        M.plan_mm(xg, w, p, out=out2)

    def pulled():
        epoch[0] += 1
        C.gemm_grouped_dev_pull(stage, w, out, p.tiles, p.ntiles, peers, H, index, p.offsets[-1:], flags,
                                epoch[0], False)

    used = int(p.offsets[-1])
    flops = 2.0 * T * k * H * N
    rows = []
    for name, fn in (("gather_then_grouped_gemm", gathered), ("pull_staged_grouped_gemm", pulled)):
        ms = median_ms(time_cuda(fn, iters=a.iters, warmup=3))
        rows.append({"variant": name, "ms": round(ms, 4), "TFLOP/s": round(flops / ms / 1e9, 1)})
        print(json.dumps(rows[-1]), flush=True)
    torch.cuda.synchronize()
    same = bool(torch.allclose(out[:used].float(), out2[:used].float(), atol=2e-2, rtol=2e-2))
    print(json.dumps({"outputs_match": same, "device_error": ops.check_device_error()}), flush=True)
    return rows


if __name__ == "__main__":
    main()
