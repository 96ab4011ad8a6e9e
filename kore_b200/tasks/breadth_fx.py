"""Breadth families, part 4: fused epilogues, quantisation and GEMM layouts.

* fx (fused): residual + RMSNorm + fp8 quantisation, bias + GELU + residual,
  SwiGLU + down-projection input scaling, RoPE + q/k RMSNorm, softmax +
  dropout-free attention-probability scaling, GEGLU, ReGLU, add + LayerNorm,
  scaled masked softmax, logit soft-cap + log-softmax, RMSNorm + gating (x *
  silu(z)), bias + SiLU + mul;
* qx (quantisation): per-channel int8, per-token int8, per-tensor fp8 e5m2,
  per-token fp8 e4m3 (dynamic), group-wise int4 (pack two nibbles per byte),
  NF4-style codebook dequantisation, MX-fp4 block dequantisation (32-element
  blocks with a power-of-two scale), SmoothQuant activation scaling, int8
  dequantisation with per-channel scales;
* gemm layouts: A^T B, A B^T, A^T B^T, GEMV (M = 1), skinny (M = 16 .. 64),
  K-heavy, rank-k update, strided batched with broadcast weights.

Module-level PyTorch definitions as oracle (fp32), vendor baseline (task
dtype) and seed. Reference parity: task dirs ``genb_fx_*``, ``genb_qx_*``,
``genb_gemm_*`` of the reference, written from the operator definitions.
"""
from __future__ import annotations

import math
from typing import Callable, List

import torch
import torch.nn.functional as F

from .spec import OpSpec, _gen, _randn

FP8_MAX = 448.0
E5M2_MAX = 57344.0


def _fp32_of(f):
    return lambda *x: f(*(t.float() if t.is_floating_point() else t for t in x))


def _seed_for(entry: str, args: str, fn: Callable) -> str:
    return (f"from kore_b200.tasks.breadth_fx import {fn.__name__} as _ref\n\n\n"
            f"def {entry}({args}):\n    return _ref({args})\n")


# ============================================================================= fused
def mk_fx(d, s, dev, dt):
    M, N = d["M"], d["N"]
    x = _randn((M, N), s, dev, dt)
    r = _randn((M, N), s + 1, dev, dt)
    w = (1 + 0.1 * _randn((N,), s + 2, dev, torch.float32)).to(dt)
    b = (0.1 * _randn((N,), s + 3, dev, torch.float32)).to(dt)
    return x, r, w, b


def _rms(x, w, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def fx_residual_rmsnorm_fp8(x, r, w, b):
    """h = x + r; y = rmsnorm(h) quantised to e4m3 with a per-row scale;
    returns dequantised y and h."""
    h = x + r
    y = _rms(h, w)
    sc = y.abs().amax(-1, keepdim=True).clamp_min(1e-12) / FP8_MAX
    q = (y / sc).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).float() * sc
    return torch.cat([q, h], -1)


def fx_bias_gelu_residual(x, r, w, b):
    return F.gelu(x + b, approximate="tanh") + r


def fx_bias_silu_mul(x, r, w, b):
    return F.silu(x + b) * r


def fx_geglu(x, r, w, b):
    return F.gelu(x) * r


def fx_reglu(x, r, w, b):
    return torch.relu(x) * r


def fx_add_layernorm(x, r, w, b):
    return F.layer_norm(x + r, x.shape[-1:], w, b, 1e-5)


def fx_rmsnorm_gated(x, r, w, b):
    """Mamba-2 style: rmsnorm(x * silu(z)) with z = r."""
    return _rms(x * F.silu(r), w)


def fx_scaled_masked_softmax(x, r, w, b, scale=0.125):
    mask = r > 1.5
    return torch.softmax((x * scale).masked_fill(mask, float("-inf")), -1)


def fx_softcap_logsoftmax(x, r, w, b, cap=30.0):
    return torch.log_softmax(cap * torch.tanh(x / cap), -1)


def fx_swiglu_scaled(x, r, w, b):
    """SwiGLU output scaled per column (the down-projection's input scale)."""
    return F.silu(x) * r * w


def fx_residual_scale_add(x, r, w, b, alpha=0.5):
    return alpha * x + r * w + b


def mk_fx_rope(d, s, dev, dt):
    S, H = d["S"], d["H"]
    q = _randn((S, H, 128), s, dev, dt)
    w = (1 + 0.1 * _randn((128,), s + 1, dev, torch.float32)).to(dt)
    pos = torch.arange(S, device=dev, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128))
    ang = pos[:, None] * inv[None]
    return q, w, ang.cos().to(dt), ang.sin().to(dt)


def fx_qknorm_rope(q, w, cos, sin):
    x = _rms(q, w)
    x1, x2 = x[..., :64], x[..., 64:]
    c, s_ = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_], -1)


FUSED = [fx_residual_rmsnorm_fp8, fx_bias_gelu_residual, fx_bias_silu_mul, fx_geglu, fx_reglu, fx_add_layernorm,
         fx_rmsnorm_gated, fx_scaled_masked_softmax, fx_softcap_logsoftmax, fx_swiglu_scaled, fx_residual_scale_add]


# ============================================================================= quantisation
def mk_q(d, s, dev, dt):
    x = _randn((d["M"], d["N"]), s, dev, dt)
    a = (0.5 + torch.rand((d["N"],), generator=_gen(s + 1, dev), device=dev)).to(dt)
    return x, a


def qx_int8_per_channel(x, a):
    sc = x.abs().amax(0, keepdim=True).clamp_min(1e-12) / 127
    return torch.round(x / sc).clamp(-127, 127) * sc


def qx_int8_per_token(x, a):
    sc = x.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 127
    return torch.round(x / sc).clamp(-127, 127) * sc


def qx_fp8_e5m2_per_tensor(x, a):
    sc = x.abs().amax().clamp_min(1e-12) / E5M2_MAX
    return (x / sc).to(torch.float8_e5m2).float() * sc


def qx_fp8_e4m3_per_token(x, a):
    sc = x.abs().amax(-1, keepdim=True).clamp_min(1e-12) / FP8_MAX
    return (x / sc).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).float() * sc


def qx_int4_group128(x, a):
    """Symmetric int4 with one scale per 128 columns; returns the dequantised
    tensor (the packed form is two nibbles per byte)."""
    M, N = x.shape
    g = x.reshape(M, N // 128, 128)
    sc = g.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 7
    return (torch.round(g / sc).clamp(-8, 7) * sc).reshape(M, N)


_NF4 = None


def _nf4_levels(device):
    """16 levels at the quantiles of a standard normal, scaled to [-1, 1]
    (the NormalFloat-4 construction), including an exact zero."""
    global _NF4
    if _NF4 is None:
        normal = torch.distributions.Normal(0.0, 1.0)
        pos = normal.icdf(torch.linspace(0.5, 0.9677, 9)[1:])
        neg = -normal.icdf(torch.linspace(0.5, 0.9677, 8)[1:])
        lv = torch.cat([neg.flip(0), torch.zeros(1), pos])
        _NF4 = lv / lv.abs().max()
    return _NF4.to(device)


def qx_nf4_roundtrip(x, a):
    M, N = x.shape
    g = x.reshape(M, N // 64, 64)
    absmax = g.abs().amax(-1, keepdim=True).clamp_min(1e-12)
    lv = _nf4_levels(x.device)
    idx = ((g / absmax)[..., None] - lv).abs().argmin(-1)
    return (lv[idx] * absmax).reshape(M, N)


def qx_mxfp4_roundtrip(x, a):
    """MX-fp4 (e2m1 values, one power-of-two scale per 32 elements)."""
    M, N = x.shape
    g = x.reshape(M, N // 32, 32)
    e = torch.floor(torch.log2(g.abs().amax(-1, keepdim=True).clamp_min(1e-30))) - 2
    sc = torch.exp2(e)
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], device=x.device)
    y = (g / sc).clamp(-6, 6)
    idx = (y.abs()[..., None] - vals).abs().argmin(-1)
    return (torch.sign(y) * vals[idx] * sc).reshape(M, N)


def qx_smoothquant_scale(x, a, alpha=0.5):
    """Per-column migration scale s = max|x|^alpha / max|w|^(1-alpha) (the
    weight maxima given as ``a``), applied to the activations."""
    s_ = x.abs().amax(0).clamp_min(1e-5).pow(alpha) / a.clamp_min(1e-5).pow(1 - alpha)
    return x / s_


def qx_int8_dequant(x, a):
    q = torch.round(x * 20).clamp(-127, 127)
    return q * (a / 20)


QUANT = [qx_int8_per_channel, qx_int8_per_token, qx_fp8_e5m2_per_tensor, qx_fp8_e4m3_per_token, qx_int4_group128,
         qx_nf4_roundtrip, qx_mxfp4_roundtrip, qx_smoothquant_scale, qx_int8_dequant]


# ============================================================================= gemm layouts
def mk_ab(d, s, dev, dt):
    M, N, K = d["M"], d["N"], d["K"]
    return _randn((M, K), s, dev, dt, K ** -0.25), _randn((K, N), s + 1, dev, dt, K ** -0.25)


def gemm_at_b(a, b):
    return a.t().contiguous().t() @ b                    # A stored K-major transposed


def gemm_a_bt(a, b):
    return a @ b.t().contiguous().t()


def gemm_at_bt(a, b):
    return (b.t() @ a.t()).t()


def gemm_rank_k_update(a, b):
    """C = A B + A[:, :64] B[:64] (a rank-64 correction fused into one GEMM)."""
    return a @ b + a[:, :64] @ b[:64]


def gemm_gemv(a, b):
    return a[:1] @ b


def mk_bcast(d, s, dev, dt):
    B, M, N, K = d["B"], d["M"], d["N"], d["K"]
    return _randn((B, M, K), s, dev, dt, K ** -0.25), _randn((K, N), s + 1, dev, dt, K ** -0.25)


def gemm_batched_broadcast_w(a, b):
    return a @ b


GEMM_LAYOUTS = [gemm_at_b, gemm_a_bt, gemm_at_bt, gemm_rank_k_update, gemm_gemv]
GEMM_SHAPES = {"square4k": (4096, 4096, 4096), "skinny16": (16, 8192, 8192), "skinny64": (64, 14336, 4096),
               "kheavy": (1024, 1024, 32768), "wide": (2048, 28672, 4096)}


def build() -> List[OpSpec]:
    out: List[OpSpec] = []
    for dt in ("bf16", "fp16"):
        for (M, N) in ((8192, 5120), (4096, 8192)):
            sh = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": M, "N": N}, "validation": [{"M": 333, "N": 2048}]}
            for fn in FUSED:
                out.append(OpSpec(f"genb_fx_{fn.__name__[3:]}_m{M}n{N}_{dt}", "fused_elementwise", "fused", mk_fx,
                                  _fp32_of(fn), fn, _seed_for("fused", "x, r, w, b", fn), sh, "fused", dt))
            for fn in QUANT:
                out.append(OpSpec(f"genb_qx_{fn.__name__[3:]}_m{M}n{N}_{dt}", "quant", "quant", mk_q, _fp32_of(fn),
                                  fn, _seed_for("quant", "x, a", fn), sh, "quant", dt))
        for H in (32, 40, 64):
            sh = {"minimal": {"S": 16, "H": 2}, "primary": {"S": 8192, "H": H}, "validation": []}
            out.append(OpSpec(f"genb_fx_qknorm_rope_h{H}_{dt}", "rope", "fused", mk_fx_rope, _fp32_of(fx_qknorm_rope),
                              fx_qknorm_rope, _seed_for("fused", "q, w, cos, sin", fx_qknorm_rope),
                              {**sh, "primary": {**sh["primary"], "D": 128}, "minimal": {**sh["minimal"], "D": 128}},
                              "fused", dt))
        for nm, (M, N, K) in GEMM_SHAPES.items():
            sh = {"minimal": {"M": 64, "N": 128, "K": 128}, "primary": {"M": M, "N": N, "K": K}, "validation": []}
            for fn in GEMM_LAYOUTS:
                if fn is gemm_gemv and nm != "square4k":
                    continue
                out.append(OpSpec(f"genb_gemm_{fn.__name__[5:]}_{nm}_{dt}", "gemm", "gemm", mk_ab, _fp32_of(fn), fn,
                                  _seed_for("gemm", "a, b", fn), sh, "gemm_ext", dt))
        shb = {"minimal": {"B": 2, "M": 32, "N": 64, "K": 64}, "primary": {"B": 16, "M": 512, "N": 4096, "K": 4096},
               "validation": []}
        out.append(OpSpec(f"genb_gemm_batched_broadcast_w_{dt}", "batched_gemm", "gemm", mk_bcast,
                          _fp32_of(gemm_batched_broadcast_w), gemm_batched_broadcast_w,
                          _seed_for("gemm", "a, b", gemm_batched_broadcast_w), shb, "gemm_ext", dt))
    return out
