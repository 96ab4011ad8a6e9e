"""tcgen05 flash attention vs torch SDPA (cuDNN / flash backends) on the
Qwen3-14B shape: causal, 40 Q / 8 KV heads, head_dim 128.

    python -m kore_b200.bench.attn_bench [--seq 8192]
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from kore_b200.bench.timing import median_ms, time_cuda
from kore_b200.ops import attention as attn


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--hq", type=int, default=40)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    T, D = a.seq, 128
    torch.manual_seed(0)
    qk = torch.randn(T, (a.hq + a.hkv) * D, device="cuda").bfloat16()
    v = torch.randn(T, a.hkv, D, device="cuda").bfloat16()
    q = qk[:, : a.hq * D].view(T, a.hq, D)
    k = qk[:, a.hq * D:].view(T, a.hkv, D)
    cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
    o, lse = attn.attn_fwd(q, k, v, cu, T)
    do = torch.randn_like(o)
    fl_fwd = 4.0 * T * T * D * a.hq / 2
    fwd = median_ms(time_cuda(lambda: attn.attn_fwd(q, k, v, cu, T), a.iters))
    bwd = median_ms(time_cuda(lambda: attn.attn_bwd(do, q, k, v, o, lse, cu, T), a.iters))
    qs, ks, vs = (x.transpose(0, 1).unsqueeze(0) for x in (q, k, v))
    sd = lambda: torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True,
                                                                   enable_gqa=True)
    sfwd = median_ms(time_cuda(sd, a.iters))
    qr, kr, vr = (x.detach().clone().requires_grad_(True) for x in (qs, ks, vs))
    out = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr, is_causal=True, enable_gqa=True)
    g = torch.randn_like(out)
    sbwd = median_ms(time_cuda(lambda: torch.autograd.grad(out, (qr, kr, vr), g, retain_graph=True),
                               a.iters))
    r = {"seq": T, "fwd_ms": fwd, "bwd_ms": bwd, "fwd_tflops": fl_fwd / fwd / 1e9,
         "bwd_tflops": 2.5 * fl_fwd / bwd / 1e9, "sdpa_fwd_ms": sfwd, "sdpa_bwd_ms": sbwd,
         "sdpa_fwd_tflops": fl_fwd / sfwd / 1e9, "sdpa_bwd_tflops": 2.5 * fl_fwd / sbwd / 1e9}
    print(json.dumps(r))


if __name__ == "__main__":
    main()
