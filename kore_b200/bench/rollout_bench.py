"""Decode-step benchmark of the rollout engine (CUDA-graph decode loop).

    python -m kore_b200.bench.rollout_bench [--batch 64] [--ctx 4096] [--layers 0]

Times one replay of the captured decode step for ``batch`` sequences whose KV
history is ``ctx`` tokens, plus its parts in isolation (the decode GEMMs at
M = batch, the paged attention, the sampler). Prints one JSON line with the
step time, the bytes a step must read (weights + KV history) and the achieved
fraction of the measured HBM bandwidth (MEASURED_PEAKS.json).
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from kore_b200 import ops
from kore_b200.analysis.rooflines import measured_peaks
from kore_b200.bench.timing import median_ms, time_cuda
from kore_b200.engine.multiturn import DecodeGraph
from kore_b200.engine.rollout import RolloutEngine
from kore_b200.models import PRESETS, Qwen3Weights


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-14b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--nsplit", type=int, default=4)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    cfg = PRESETS[args.model]()
    if args.layers:
        cfg.num_hidden_layers = args.layers
    torch.manual_seed(0)
    w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    B, L, ps = args.batch, args.ctx, 64
    pages_per = (L + 1 + ps - 1) // ps + 1
    eng = RolloutEngine(w, max_batch=B, page_size=ps, num_pages=B * pages_per, max_seq_len=L + 2 * ps)
    for t in eng.cache.k + eng.cache.v:
        t.normal_(0, 1)
    g = DecodeGraph(eng, B, 1 << 20, nsplit=args.nsplit, temperature=1.0)
    for i in range(B):
        g.bt[i, :pages_per] = torch.arange(i * pages_per, (i + 1) * pages_per, dtype=torch.int32)
    g.pos.fill_(L)
    g.active.fill_(False)   # keep the position fixed: every replay decodes at context L
    g.budget.fill_(1 << 30)
    g.tok.random_(0, cfg.vocab_size)
    g.step()                # capture
    out = {"batch": B, "ctx": L, "layers": cfg.num_hidden_layers, "nsplit": args.nsplit}
    out["step_ms"] = median_ms(time_cuda(g.step, args.iters, flush_l2=False))
    wbytes = sum(b.numel() * b.element_size() for b in w.bufs)
    kvbytes = B * (L + 1) * eng.kv_bytes_per_token()
    out["weights_gb"] = round(wbytes / 1e9, 2)
    out["kv_gb"] = round(kvbytes / 1e9, 2)
    peaks = measured_peaks() or {}
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * 1e9
    out["hbm_floor_ms"] = round((wbytes + kvbytes) / hbm * 1e3, 3)
    out["fraction_of_measured_hbm"] = round(out["hbm_floor_ms"] / out["step_ms"], 3)
    # parts in isolation
    x = torch.randn(B, cfg.hidden_size, device="cuda").bfloat16()
    W1 = w.views(1)
    parts = {}
    for name, a, wt in (("qkv", x, W1["qkv"]), ("o", torch.randn(B, cfg.q_dim, device="cuda").bfloat16(), W1["o"]),
                        ("gate_up", x, W1["gate_up"]),
                        ("down", torch.randn(B, cfg.intermediate_size, device="cuda").bfloat16(), W1["down"]),
                        ("lm_head", x, w.lm_head_weight())):
        ms = median_ms(time_cuda(lambda: ops.mm(a, wt), args.iters))
        parts[name + "_ms"] = round(ms, 4)
        parts[name + "_gbs"] = round(wt.numel() * 2 / ms / 1e6, 1)
    q = torch.randn(B, eng.hq, eng.D, device="cuda").bfloat16()
    lens = torch.full((B,), L + 1, dtype=torch.int32, device="cuda")
    ms = median_ms(time_cuda(lambda: eng._paged_attention(q, 0, g.bt, lens, g.qs, 1, 1 / math.sqrt(eng.D),
                                                          g.nsplit, g.part_o, g.part_ml), args.iters))
    parts["attention_ms"] = round(ms, 4)
    parts["attention_gbs"] = round(B * (L + 1) * eng.kv_bytes_per_token() / cfg.num_hidden_layers / ms / 1e6, 1)
    logits = torch.randn(B, cfg.vocab_size, device="cuda").bfloat16()
    tok = torch.empty(B, dtype=torch.long, device="cuda")
    lp = torch.empty(B, device="cuda")
    parts["sampler_ms"] = round(median_ms(time_cuda(
        lambda: ops.native().sample_tokens(logits, 1.0, 1.0, 0, 1, tok, lp), args.iters)), 4)
    out["parts"] = parts
    out["device_error"] = ops.check_device_error()
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
