"""Bandwidth of the memory-bound training kernels at Qwen3-14B shapes.

    python -m kore_b200.bench.ops_bench [--tokens 8192] [--iters 10] [--only NAME]

Times RMSNorm forward / backward (with the residual gradient), q/k RMSNorm +
RoPE forward, SwiGLU forward / backward, the fused vocabulary log-prob +
gradient (one 2,048-row chunk of the LM head's logits, overwritten in place
by the gradient) and the AdamW step over one decoder layer's MLP weights
(bf16 parameters and gradients, fp32 moments, stochastic rounding). Each is
timed with CUDA events on the launching stream after warm-up, with L2
flushed between iterations; the achieved figure is the kernel's compulsory
HBM bytes (each operand read or written once) over the median time, also
given as a fraction of the measured copy bandwidth when MEASURED_PEAKS.json
is present (else the pool's 6.65 TB/s fallback).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops
from ..ops import reference as ref
from .timing import median_ms, time_cuda

H, HQ, HKV, D, FF, V = 5120, 40, 8, 128, 17408, 151936


def _peak_gbs() -> tuple[float, str]:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def cases(T: int, dev):
    bf = dict(dtype=torch.bfloat16, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    x = torch.randn(T, H, **bf)
    w = 1 + 0.1 * torch.randn(H, **bf)
    rstd = torch.empty(T, **f32)
    out = torch.empty_like(x)
    dy, dres = torch.randn_like(x), torch.randn_like(x)
    dw = torch.zeros(H, **f32)
    yield ("rmsnorm_fwd", lambda: ops.rmsnorm_fwd(x, w, 1e-6, rstd=rstd, out=out), 2 * T * H * 2 + T * 4)
    yield ("rmsnorm_bwd", lambda: ops.rmsnorm_bwd(dy, x, w, rstd, dres=dres, dw=dw, out=out),
           4 * T * H * 2 + T * 4)
    del dy, dres
    qkv = torch.randn(T, (HQ + 2 * HKV) * D, **bf)
    qw, kw = torch.ones(D, **bf), torch.ones(D, **bf)
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    cos, sin = ref.rope_tables(max(T, 8192), D, 1e6, dev)
    qk = torch.empty(T, (HQ + HKV) * D, **bf)
    qrs = torch.empty(T, HQ + HKV, **f32)
    yield ("qk_norm_rope_fwd", lambda: ops.qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, HQ, HKV, 1e-6,
                                                            rstd=qrs, out=qk),
           2 * T * (HQ + HKV) * D * 2)
    del qkv, qk
    gu = torch.randn(T, 2 * FF, **bf)
    h = torch.empty(T, FF, **bf)
    dh = torch.randn(T, FF, **bf)
    dgu = torch.empty_like(gu)
    yield ("swiglu_fwd", lambda: ops.swiglu_fwd(gu, out=h), T * 3 * FF * 2)
    yield ("swiglu_bwd", lambda: ops.swiglu_bwd(dh, gu, dgu), T * 5 * FF * 2)
    del gu, h, dh, dgu
    R = 2048
    logits = torch.randn(R, V, **bf)
    tg = torch.randint(0, V, (R,), device=dev)
    coef = torch.full((R,), 1.0 / R, **f32)
    yield ("logprob_grad", lambda: ops.logprob(logits, tg, coef=coef, write_grad=True), 2 * R * V * 2 + R * 16)
    del logits
    n = 3 * H * FF
    p = torch.randn(n, **bf) * 0.02
    g = torch.randn(n, **bf) * 1e-3
    m, v = torch.zeros(n, **f32), torch.zeros(n, **f32)
    yield ("adamw_bf16_sr", lambda: ops.adamw_step(p, g, m, v, lr=1e-5, wd=0.1, step=3), n * (2 * 2 + 2 + 2 * 8))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--only", default="")
    a = ap.parse_args(argv)
    ops.native()
    peak, kind = _peak_gbs()
    rows = []
    for name, fn, nbytes in cases(a.tokens, torch.device("cuda")):
        if a.only and a.only not in name:
            continue
        ms = median_ms(time_cuda(fn, iters=a.iters, warmup=3))
        gbs = nbytes / ms / 1e6
        rows.append({"kernel": name, "ms": round(ms, 4), "bytes": int(nbytes), "GB/s": round(gbs, 1),
                     f"frac_of_{kind}_hbm": round(gbs / peak, 3)})
        print(json.dumps(rows[-1]), flush=True)
    assert ops.check_device_error() == 0
    return rows


if __name__ == "__main__":
    main()
