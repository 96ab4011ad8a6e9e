"""Device-timed comparison of the fused peer-memory paths with their NCCL
baselines, each reported against its roofline (run under torchrun, >= 2 GPUs):

    python -m torch.distributed.run --nproc-per-node N -m kore_b200.parallel.collective_bench

(b) ZeRO-2 optimizer step on a flat parameter set: NCCL reduce-scatter +
    sharded AdamW + all-gather, versus ONE fused kernel per unit that reads
    the peers' gradient shards over NVLink, updates, and stores the new
    parameters into every peer. Roofline: the slower of the NVLink bytes per
    direction per GPU (2 P (N-1)/N each way) at the measured peer bandwidth
    and the local HBM bytes at the measured copy bandwidth.
(c) tensor-parallel all-gather -> GEMM (the GEMM's CTAs stage each peer's
    row blocks into local memory once and flag them; tiles start on local
    rows) versus NCCL all-gather + GEMM, and GEMM ->
    reduce-scatter (P2P-store epilogue + fused reduce) versus GEMM + NCCL
    reduce-scatter. Roofline: max(FLOPs / measured bf16 peak, NVLink bytes /
    link bandwidth).
(d) MoE dispatch fused with the gate/up grouped GEMM (the GEMM pulls its
    receive rows from the peers in its prologue) versus P2P push + GEMM and
    versus NCCL all-to-all + GEMM; pull-combine with routing weights and
    residual versus NCCL all-to-all back. Rooflines: max(GEMM FLOPs at the
    measured bf16 peak, token rows over NVLink at link bandwidth).

Every number is CUDA-event time on the launching stream after warm-up, max
over ranks. Prints one JSON line per path from rank 0.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_BPS = 770e9      # measured peer copy per direction per GPU on this pool


def _peaks():
    from ..analysis.rooflines import resolve_peaks
    p = resolve_peaks()
    return p["hbm_bytes_per_s"], p["bf16_flops_per_s"]


def _time(fn, ctx, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ctx.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return ctx.max_over_ranks(a.elapsed_time(b) / iters)


def bench_optimizer(ctx, params: int, units: int) -> dict:
    from .. import ops
    from .symmetric import SymmetricHeap
    C = ops.native()
    W, r = ctx.world, ctx.rank
    U = (params // units) // (128 * W) * (128 * W)
    s = U // W
    heap = SymmetricHeap(ctx, 2 * 2 * U * units + (1 << 20))
    P = [heap.alloc(U)[1].normal_(0, 0.02) for _ in range(units)]
    G = [heap.alloc(U)[1].normal_(0, 1e-3) for _ in range(units)]
    m = [torch.zeros(s, device="cuda") for _ in range(units)]
    v = [torch.zeros(s, device="cuda") for _ in range(units)]
    master = [P[u][r * s:(r + 1) * s].float() for u in range(units)]
    p_off = [heap.offset_of(t) for t in P]
    g_off = [heap.offset_of(t) for t in G]
    step = [0]

    def fused():
        step[0] += 1
        heap.barrier()
        for u in range(units):
            C.symm_adamw_bcast(heap.id, p_off[u], g_off[u], s, 1.0, master[u], m[u], v[u], 1e-5, 0.9, 0.95, 1e-8,
                               0.0, step[0], None, 0.0, u)
        heap.barrier()

    gshard = [torch.empty(s, dtype=torch.bfloat16, device="cuda") for _ in range(units)]

    def nccl():
        step[0] += 1
        for u in range(units):
            dist.reduce_scatter_tensor(gshard[u], G[u], group=ctx.group)
            ops.adamw_step(P[u][r * s:(r + 1) * s], gshard[u], m[u], v[u], lr=1e-5, b1=0.9, b2=0.95, step=step[0],
                           master=master[u])
            dist.all_gather_into_tensor(P[u], P[u][r * s:(r + 1) * s], group=ctx.group)

    t_f = _time(fused, ctx)
    t_n = _time(nccl, ctx)
    hbm, _ = _peaks()
    Ptot = U * units
    link = 2.0 * Ptot * (W - 1) / W                       # bytes per direction per GPU
    local = Ptot / W * (2 + 4 * 2 * 2 + 4 * 2) + 2.0 * Ptot * (W - 1) / W * 2   # shard state r/w + peer traffic landing in HBM
    t_roof = max(link / LINK_BPS, local / hbm) * 1e3
    return {"path": "b_rs_adamw_ag", "world": W, "params": Ptot, "fused_ms": t_f, "nccl_ms": t_n,
            "roofline_ms": t_roof, "fused_frac_of_roofline": t_roof / t_f, "nccl_frac_of_roofline": t_roof / t_n,
            "speedup_vs_nccl": t_n / t_f}


def bench_tp(ctx, rows: int, K: int, N_local: int) -> list:
    from .. import ops
    from .symmetric import SymmetricHeap
    C = ops.native()
    W, r = ctx.world, ctx.rank
    M = rows * W
    heap = SymmetricHeap(ctx, (rows * K + W * rows * K) * 2 + (1 << 20))
    o_a, a_loc = heap.alloc(rows * K)
    o_s, slots = heap.alloc(W * rows * K)
    a_loc.normal_()
    a_peers = C.symm_peer_addrs(heap.id, o_a)
    s_peers = C.symm_peer_addrs(heap.id, o_s)
    w_col = torch.randn(N_local, K, device="cuda", dtype=torch.bfloat16) * 0.02   # column-parallel shard
    w_row = torch.randn(K, N_local, device="cuda", dtype=torch.bfloat16) * 0.02   # row-parallel shard [H, F/W]
    out = torch.empty(M, N_local, device="cuda", dtype=torch.bfloat16)
    gathered = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    x_full = torch.randn(M, N_local, device="cuda", dtype=torch.bfloat16)
    rs_out = torch.empty(rows, K, device="cuda", dtype=torch.bfloat16)
    stage = torch.empty(M * K, device="cuda", dtype=torch.bfloat16)
    flags = torch.zeros(M // 64, device="cuda", dtype=torch.int32)
    epoch = [0]
    full = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    x_res = torch.zeros(rows, K, device="cuda", dtype=torch.bfloat16)

    def ag_fused():
        heap.barrier()
        epoch[0] += 1
        C.gemm_tp_bf16(None, a_peers, K, M, w_col, out, [], 0, rows, r, stage, flags, epoch[0])
        heap.barrier()            # peers finished reading my rows before they change

    def ag_nccl():
        dist.all_gather_into_tensor(gathered, a_loc.view(rows, K), group=ctx.group)
        ops.mm(gathered, w_col, out=out)

    def rs_fused():
        heap.barrier()
        C.gemm_tp_bf16(x_full, [], 0, M, w_row, None, s_peers, K, rows, r)
        heap.barrier()
        C.tp_reduce_norm(slots, W, rows, x_res, None, None, 1e-6)

    def rs_nccl():
        ops.mm(x_full, w_row, out=full)
        dist.reduce_scatter_tensor(rs_out, full, group=ctx.group)

    hbm, peak = _peaks()
    res = []
    for name, f_fused, f_nccl, flops, link in (
            ("c_allgather_gemm", ag_fused, ag_nccl, 2.0 * M * N_local * K, 2.0 * rows * (W - 1) * K),
            ("c_gemm_reducescatter", rs_fused, rs_nccl, 2.0 * M * K * N_local, 2.0 * rows * (W - 1) * K)):
        tf, tn = _time(f_fused, ctx), _time(f_nccl, ctx)
        roof = max(flops / peak, link / LINK_BPS) * 1e3
        res.append({"path": name, "world": W, "M": M, "K": K, "N_local": N_local, "fused_ms": tf, "nccl_ms": tn,
                    "roofline_ms": roof, "fused_frac_of_roofline": roof / tf, "nccl_frac_of_roofline": roof / tn,
                    "speedup_vs_nccl": tn / tf})
    return res


def bench_ep(ctx, tokens: int) -> list:
    """(d) MoE for the Qwen3-Coder-30B-A3B shape (H 2048, 128 experts, top-8,
    expert FFN 768): dispatch + the gate/up grouped GEMM, three ways:
    pull (index push, one barrier, the GEMM stages its receive rows from the
    peers in its prologue), push (P2P scatter, barrier, pad zeroing, grouped
    GEMM) and NCCL (all-to-all of the rows, then the same grouped GEMM);
    then the combine: fused pull-combine with the routing weights and
    residual versus NCCL all-to-all back + weighted sum. Roofline of dispatch
    + GEMM: max(GEMM FLOPs at the measured bf16 peak, token rows over NVLink
    at link bandwidth); of the combine: the rows over NVLink."""
    from .. import ops
    from ..models.config import qwen3_coder_30b_a3b
    from ..ops import moe as moe_ops
    from .ep import FusedExpertParallel
    from .symmetric import SymmetricHeap
    C = ops.native()
    cfg = qwen3_coder_30b_a3b()
    W, r = ctx.world, ctx.rank
    E, k, H, I = cfg.num_experts, cfg.num_experts_per_tok, cfg.hidden_size, cfg.moe_intermediate_size
    El = E // W
    cap = int(2.0 * tokens * k)
    heap = SymmetricHeap(ctx, FusedExpertParallel.heap_bytes(cfg, cap, "pull") + (1 << 20))
    fep = FusedExpertParallel(ctx, cfg, r * El, (r + 1) * El, heap, cap, dispatch="pull")
    fep.k = k
    g = torch.Generator(device="cuda").manual_seed(11 + r)
    logits = torch.randn(tokens, E, device="cuda", generator=g)
    wts, idx = torch.softmax(logits, -1).topk(k, -1)
    wts = (wts / wts.sum(-1, keepdim=True)).float().contiguous()
    idx = idx.int().contiguous()
    x = torch.randn(tokens, H, device="cuda", dtype=torch.bfloat16)
    wgu = torch.randn(El, 2 * I, H, device="cuda", dtype=torch.bfloat16) * 0.02
    pl = fep._plan(idx)
    y = torch.empty_like(x)
    _, peak_flops = _peaks()
    # NCCL arm: rows grouped by destination rank; split sizes exchanged once, outside the timing
    dst_rank = pl["dst_rank"]
    order = torch.argsort(dst_rank.long(), stable=True)
    send = torch.bincount(dst_rank.long(), minlength=W)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=ctx.group)
    ss, rs_ = send.tolist(), recv.tolist()
    rbuf = torch.empty(sum(rs_), H, device="cuda", dtype=torch.bfloat16)
    back = torch.empty(tokens * k, H, device="cuda", dtype=torch.bfloat16)
    src_row = torch.arange(tokens * k, device="cuda") // k
    xp = fep.recv[: fep.cap * H].view(fep.cap, H)
    gu = torch.empty(fep.cap, 2 * I, device="cuda", dtype=torch.bfloat16)
    Wd = {"experts_gate_up": wgu}

    def disp_pull():
        fep._pull_and_up(Wd, x, pl)

    def disp_push():
        fep.dispatch = "push"
        fep._dispatch_and_up(Wd, x, pl)
        fep.dispatch = "pull"

    def disp_nccl():
        sbuf = x.index_select(0, src_row[order])
        dist.all_to_all_single(rbuf, sbuf, rs_, ss, group=ctx.group)
        moe_ops.plan_mm(xp, wgu, pl["plan"], out=gu)

    def comb_fused():
        heap.barrier()
        C.symm_ep_gather(heap.id, fep.o_y, dst_rank.view(tokens, k), pl["dst_row"].view(tokens, k), wts, x, y,
                         None, None, H)

    def comb_nccl():
        dist.all_to_all_single(back, rbuf, ss, rs_, group=ctx.group)
        rows = torch.empty_like(back)
        rows[order] = back
        torch.add(x, (rows.view(tokens, k, H).float() * wts[..., None]).sum(1).to(x.dtype), out=y)

    # the pulled receive rows and GEMM output equal the pushed ones
    fep.dispatch = "push"
    xp_push, gu_push = fep._dispatch_and_up(Wd, x, pl)
    xp_push, gu_push = xp_push.clone(), gu_push.clone()
    fep.dispatch = "pull"
    xp_pull, gu_pull = fep._pull_and_up(Wd, x, pl)
    used = int(pl["plan"].offsets[-1])
    same = bool(torch.equal(xp_pull[:used], xp_push[:used]) and torch.equal(gu_pull[:used], gu_push[:used]))
    link = 2.0 * tokens * k * H * (W - 1) / W
    flops = 2.0 * tokens * k * H * 2 * I              # gate/up GEMM rows received per rank (balanced routing)
    res = []
    tp, tpush, tn = _time(disp_pull, ctx), _time(disp_push, ctx), _time(disp_nccl, ctx)
    roof = max(link / LINK_BPS, flops / peak_flops) * 1e3
    res.append({"path": "d_moe_dispatch_gateup", "world": W, "tokens": tokens, "H": H, "topk": k,
                "pull_fused_ms": tp, "push_ms": tpush, "nccl_ms": tn, "roofline_ms": roof,
                "pull_frac_of_roofline": roof / tp, "push_frac_of_roofline": roof / tpush,
                "nccl_frac_of_roofline": roof / tn, "pull_speedup_vs_nccl": tn / tp,
                "pull_speedup_vs_push": tpush / tp, "pull_equals_push": same})
    tf, tn = _time(comb_fused, ctx), _time(comb_nccl, ctx)
    roof = link / LINK_BPS * 1e3
    res.append({"path": "d_moe_combine", "world": W, "tokens": tokens, "H": H, "topk": k, "fused_ms": tf,
                "nccl_ms": tn, "roofline_ms": roof, "fused_frac_of_roofline": roof / tf,
                "nccl_frac_of_roofline": roof / tn, "speedup_vs_nccl": tn / tf})
    from ..ops import check_device_error
    res[-1]["device_error"] = check_device_error()
    return res


def main(argv=None) -> int:
    from .dist import init_distributed
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=int, default=2_000_000_000)
    ap.add_argument("--units", type=int, default=8)
    ap.add_argument("--rows", type=int, default=2048, help="TP rows per rank")
    ap.add_argument("--ep-tokens", type=int, default=8192, help="MoE tokens per rank")
    ap.add_argument("--only", default="", choices=["", "optimizer", "tp", "ep"])
    a = ap.parse_args(argv)
    ctx = init_distributed()
    W = ctx.world
    out = []
    if a.only in ("", "optimizer"):
        out.append(bench_optimizer(ctx, a.params, a.units))
    if a.only in ("", "tp"):
        out += bench_tp(ctx, a.rows, 5120, (40 + 16) * 128 // W)    # QKV projection of the 14B model
        out += bench_tp(ctx, a.rows, 5120, 2 * 17408 // W)          # gate|up projection
    if a.only in ("", "ep"):
        out += bench_ep(ctx, a.ep_tokens)
    if ctx.is_main:
        for r in out:
            print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()}), flush=True)
    ctx.barrier()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
