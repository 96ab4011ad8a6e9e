"""MoE kernels (grouped tcgen05 GEMM, routing, combine) and MoE engine on the GPU."""
import pytest
import torch

from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
from kore_b200.models import Qwen3Config, Qwen3Weights
from kore_b200.models.reference_forward import forward_logprobs, leaf_buffers
from kore_b200.ops import moe

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("w_t", [True, False])
def test_grouped_gemm(w_t):
    torch.manual_seed(0)
    E, K, N = 6, 256, 384
    counts = [0, 130, 7, 256, 1, 300]
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + c)
    a = torch.randn(offs[-1], K, device="cuda").bfloat16()
    w = (torch.randn(E, N, K) if w_t else torch.randn(E, K, N)).cuda().bfloat16()
    out = torch.full((offs[-1], N), 7.0, device="cuda").bfloat16()
    moe.grouped_mm(a, w, offs, w_t=w_t, out=out)
    for e in range(E):
        s, t = offs[e], offs[e + 1]
        if t > s:
            ref = a[s:t].float() @ (w[e].float().t() if w_t else w[e].float())
            assert _rel(out[s:t], ref) < 8e-3, e


def test_route_and_combine_vs_cpu():
    torch.manual_seed(1)
    T, E, k, H = 300, 128, 8, 512
    logits = torch.randn(T, E, device="cuda")
    p, i, w = moe.route(logits, k, True)
    p2, i2, w2 = moe.route(logits.cpu(), k, True)
    assert torch.equal(i.cpu().long().sort(-1).values, i2.long().sort(-1).values)
    assert torch.allclose(w.cpu().sort(-1).values, w2.sort(-1).values, atol=1e-5)
    dw = torch.randn(T, k, device="cuda")
    assert torch.allclose(moe.route_bwd(p, i, w, dw).cpu(), moe.route_bwd(p.cpu(), i.cpu(), w.cpu(), dw.cpu()),
                          atol=1e-5)
    src, pos, offs = moe.permutation(i, E)
    yp = torch.randn(src.numel(), H, device="cuda").bfloat16()
    res = torch.randn(T, H, device="cuda").bfloat16()
    y = moe.combine(yp, pos, w, res)
    y2 = moe.combine(yp.cpu(), pos.cpu(), w.cpu(), res.cpu())
    assert _rel(y, y2) < 1e-2
    dy = torch.randn(T, H, device="cuda").bfloat16()
    ds, dwt = moe.combine_bwd(dy, yp, pos, w)
    ds2, dwt2 = moe.combine_bwd(dy.cpu(), yp.cpu(), pos.cpu(), w.cpu())
    assert _rel(ds, ds2) < 1e-2 and _rel(dwt, dwt2) < 1e-2


def test_moe_engine_gpu_vs_fp32_reference():
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, model_type="qwen3_moe",
                      num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256,
                      max_position_embeddings=1024)
    w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    g = torch.Generator().manual_seed(0)
    b = Batch.from_sequences([torch.randint(0, 1024, (n,), generator=g) for n in (200, 120)], device="cuda")
    eng = Qwen3Engine(w, grad_dtype=torch.float32)
    coef = eng.sft_coef(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=coef)
    bufs = leaf_buffers(w)
    lp, _ = forward_logprobs(w, bufs, b)
    (lp * coef).sum().backward()
    for u, (gr, r) in enumerate(zip(eng.grads, bufs)):
        rel = ((gr.float() - r.grad).norm() / (r.grad.norm() + 1e-12)).item()
        assert rel < 5e-2, (u, rel)


def test_device_plan_grouped_and_wgrad_vs_cpu():
    """Device routing plan (no host sync) equals the CPU definition; grouped
    forward and per-expert weight gradient over it match fp32."""
    from kore_b200.ops import moe
    torch.manual_seed(3)
    T, k, E, H, N = 300, 4, 16, 256, 384
    idx = torch.randint(0, E, (T, k), dtype=torch.int32)
    idx[:, 0] = 5                                  # a hot expert; some experts stay empty
    idx[idx == 7] = 8
    pc = moe.plan(idx, E)
    pg = moe.plan(idx.cuda(), E)
    assert torch.equal(pg.counts.cpu(), pc.counts) and torch.equal(pg.offsets.cpu(), pc.offsets)
    assert torch.equal(pg.pos.cpu(), pc.pos) and torch.equal(pg.src_row.cpu(), pc.src_row)
    nt = int(pc.ntiles)
    assert int(pg.ntiles) == nt and torch.equal(pg.tiles.cpu()[: 4 * nt], pc.tiles[: 4 * nt])
    x = torch.randn(T, H).bfloat16()
    w = (torch.randn(E, N, H) / H ** 0.5).bfloat16()
    xp_c = moe.plan_gather(x, pc)
    xp_g = moe.plan_gather(x.cuda(), pg)
    assert torch.equal(xp_g.cpu(), xp_c)
    y_c = moe.plan_mm(xp_c, w, pc)
    y_g = moe.plan_mm(xp_g, w.cuda(), pg)
    rows = int(pc.offsets[-1])
    assert _rel(y_g[:rows].cpu(), y_c[:rows]) < 1e-2
    dy = torch.randn(pc.rows, N).bfloat16()
    dy[pc.src_row < 0] = 0
    gw_c = torch.zeros(E, N, H, dtype=torch.float32)
    moe.plan_wgrad(dy, xp_c, pc, gw_c)
    gw_g = torch.zeros(E, N, H, dtype=torch.float32, device="cuda")
    moe.plan_wgrad(dy.cuda(), xp_g, pg, gw_g)
    assert _rel(gw_g.cpu(), gw_c) < 1e-2
    assert float(gw_g[7].abs().sum()) == 0.0          # expert without rows: untouched


def test_pull_dispatch_grouped_gemm_matches_gathered():
    """The grouped GEMM that stages its own receive rows in its prologue (the
    expert-parallel pull dispatch, here with this GPU as the only peer) gives
    the same expert outputs as gathering the rows first and running the
    grouped GEMM, on two calls in a row (the per-group flags are epoch-tagged)."""
    from kore_b200.ops import check_device_error, native
    from kore_b200.ops import moe as M
    from kore_b200.parallel.dist import DistContext
    from kore_b200.parallel.symmetric import SymmetricHeap
    C = native()
    torch.manual_seed(5)
    T, H, E, k, N = 300, 256, 8, 2, 512
    ctx = DistContext(device=torch.device("cuda"))
    idx = torch.randint(0, E, (T, k), device="cuda", dtype=torch.int32)
    w = (torch.randn(E, N, H, device="cuda") * 0.05).bfloat16()
    p = M.plan(idx, E)
    cap = (p.rows + 63) // 64 * 64
    heap = SymmetricHeap(ctx, T * H * 2 + cap * 4 + (1 << 16))
    o_tok, tok = heap.alloc(T * H)
    peers = C.symm_peer_addrs(heap.id, o_tok)
    index = torch.full((cap,), -1, dtype=torch.int32, device="cuda")
    index[: p.rows] = p.src_row                        # this rank (0) << 26 | token row; -1 = pad
    flags = torch.zeros(cap // 64, dtype=torch.int32, device="cuda")
    stage = torch.empty(cap, H, dtype=torch.bfloat16, device="cuda")
    used = int(p.offsets[-1])
    for epoch in (1, 2):
        x = torch.randn(T, H, device="cuda").bfloat16()
        tok.view(T, H).copy_(x)
        stage.fill_(float("nan"))                       # every staged row must be written, pads as zeros
        out = torch.empty(cap, N, dtype=torch.bfloat16, device="cuda")
        C.gemm_grouped_dev_pull(stage, w, out, p.tiles, p.ntiles, peers, H, index, p.offsets[-1:], flags, epoch,
                                False)
        ref = M.plan_mm(M.plan_gather(x, p), w, p)
        torch.cuda.synchronize()
        assert check_device_error() == 0
        assert torch.equal(stage[:used], M.plan_gather(x, p)[:used])
        assert torch.allclose(out[:used].float(), ref[:used].float(), atol=2e-2, rtol=2e-2)
