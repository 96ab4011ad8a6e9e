"""Operator library behind the kernel tasks (environment content).

Each :class:`OpSpec` gives, for one operation: input construction per shape
and seed, the fp32 PyTorch oracle, the vendor baseline the candidate must
beat on B200 (cuBLAS via torch.matmul, cuDNN/flash SDPA, torch fused ops),
the roofline operation name, the entry-point name the candidate module must
define, and a seed kernel (a correct but naive Triton kernel the policy
starts from). Tasks reference specs by name; the registry instantiates them
with shapes. Reference parity: the task families of kore/tasks/_genops.py
(unary / binary / reduce / fusion / gemm) and the hand-authored core tasks
(rmsnorm, softmax, silu_mul, rope, flash-attn decode/prefill, gemm, moe
routing, fp8 quant), retargeted from gfx950 to sm_100a.
"""
from __future__ import annotations

import math
from typing import Dict

import torch
import torch.nn.functional as F

from .spec import Inputs, OpSpec, _gen, _randn  # noqa: F401


# ------------------------------------------------------------------ seeds
_ROWWISE_SEED = '''import torch
import triton
import triton.language as tl


@triton.jit
def _k(X, Y, W, N, eps, BLOCK: tl.constexpr):
    row = tl.program_id(0)
    cols = tl.arange(0, BLOCK)
    m = cols < N
    x = tl.load(X + row * N + cols, mask=m, other=0.0).to(tl.float32)
    {body}
    tl.store(Y + row * N + cols, y.to(Y.dtype.element_ty), mask=m)


def {entry}(x, w=None, eps={eps}):
    M, N = x.shape
    y = torch.empty_like(x)
    ww = w if w is not None else x
    _k[(M,)](x, y, ww, N, eps, BLOCK=triton.next_power_of_2(N))
    return y
'''

_ELEMWISE_SEED = '''import torch
import triton
import triton.language as tl


@triton.jit
def _k(A, B, Y, n, BLOCK: tl.constexpr):
    i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = i < n
    a = tl.load(A + i, mask=m, other=0.0).to(tl.float32)
    b = tl.load(B + i, mask=m, other=0.0).to(tl.float32)
    {body}
    tl.store(Y + i, y.to(Y.dtype.element_ty), mask=m)


def {entry}(a, b):
    y = torch.empty_like(a)
    n = a.numel()
    _k[(triton.cdiv(n, 1024),)](a, b, y, n, BLOCK=1024)
    return y
'''

_GEMM_SEED = '''import torch
import triton
import triton.language as tl


@triton.jit
def _k(A, B, C, M, N, K, BM: tl.constexpr, BN: tl.constexpr, BK: tl.constexpr):
    pm, pn = tl.program_id(0), tl.program_id(1)
    rm = pm * BM + tl.arange(0, BM)
    rn = pn * BN + tl.arange(0, BN)
    rk = tl.arange(0, BK)
    acc = tl.zeros((BM, BN), dtype=tl.float32)
    for k in range(0, K, BK):
        a = tl.load(A + rm[:, None] * K + (k + rk)[None, :], mask=(rm[:, None] < M) & ((k + rk)[None, :] < K), other=0.0)
        b = tl.load(B + rn[None, :] * K + (k + rk)[:, None], mask=(rn[None, :] < N) & ((k + rk)[:, None] < K), other=0.0)
        acc += tl.dot(a, b)
    tl.store(C + rm[:, None] * N + rn[None, :], acc.to(C.dtype.element_ty), mask=(rm[:, None] < M) & (rn[None, :] < N))


def {entry}(a, b):
    M, K = a.shape
    N = b.shape[0]
    c = torch.empty(M, N, device=a.device, dtype=a.dtype)
    _k[(triton.cdiv(M, 64), triton.cdiv(N, 64))](a, b, c, M, N, K, BM=64, BN=64, BK=32)
    return c
'''

_DECODE_SEED = '''import torch
import triton
import triton.language as tl


@triton.jit
def _k(Q, K, V, O, S, H, KV, D: tl.constexpr, BN: tl.constexpr, scale):
    bh = tl.program_id(0)
    b, h = bh // H, bh % H
    kvh = h // (H // KV)
    d = tl.arange(0, D)
    q = tl.load(Q + (b * H + h) * D + d).to(tl.float32) * scale
    m = -float("inf")
    l = 0.0
    acc = tl.zeros((D,), dtype=tl.float32)
    for s0 in range(0, S, BN):
        s = s0 + tl.arange(0, BN)
        km = s < S
        k = tl.load(K + ((b * KV + kvh) * S + s[:, None]) * D + d[None, :], mask=km[:, None], other=0.0).to(tl.float32)
        sc = tl.sum(k * q[None, :], 1)
        sc = tl.where(km, sc, -float("inf"))
        mn = tl.maximum(m, tl.max(sc, 0))
        p = tl.exp(sc - mn)
        c = tl.exp(m - mn)
        v = tl.load(V + ((b * KV + kvh) * S + s[:, None]) * D + d[None, :], mask=km[:, None], other=0.0).to(tl.float32)
        acc = acc * c + tl.sum(p[:, None] * v, 0)
        l = l * c + tl.sum(p, 0)
        m = mn
    tl.store(O + (b * H + h) * D + d, (acc / l).to(O.dtype.element_ty))


def {entry}(q, k, v):
    B, H, D = q.shape
    KV, S = k.shape[1], k.shape[2]
    o = torch.empty_like(q)
    _k[(B * H,)](q, k, v, o, S, H, KV, D=D, BN=64, scale=1.0 / (D ** 0.5))
    return o
'''


def _rowwise(entry, body, eps=1e-6):
    return _ROWWISE_SEED.replace("{body}", body).replace("{entry}", entry).replace("{eps}", repr(eps))


def _elem(entry, body):
    return _ELEMWISE_SEED.replace("{body}", body).replace("{entry}", entry)


# ------------------------------------------------------------------ specs
def _mk_rows(d, seed, dev, dt):
    return (_randn((d["M"], d["N"]), seed, dev, dt), (1 + 0.1 * _randn((d["N"],), seed + 1, dev, torch.float32)).to(dt))


def _rmsnorm_ref(x, w, eps=1e-6):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _layernorm_ref(x, w, eps=1e-5):
    return F.layer_norm(x.float(), (x.shape[-1],), w.float(), None, eps)


def _softmax_ref(x, w=None):
    return torch.softmax(x.float(), -1)


def _mk_pair(d, seed, dev, dt):
    n = d["M"] * d["N"]
    return (_randn((n,), seed, dev, dt), _randn((n,), seed + 7, dev, dt))


def _silu_mul_ref(a, b):
    return F.silu(a.float()) * b.float()


def _gelu_tanh_ref(a, b):
    return F.gelu(a.float(), approximate="tanh") + 0 * b.float()


def _mk_gemm(d, seed, dev, dt):
    return (_randn((d["M"], d["K"]), seed, dev, dt, 0.5), _randn((d["N"], d["K"]), seed + 3, dev, dt, 0.5))


def _gemm_ref(a, b):
    return a.float() @ b.float().t()


def _mk_decode(d, seed, dev, dt):
    B, H, KV, S, D = d["B"], d["H"], d["KV"], d["S"], d["D"]
    return (_randn((B, H, D), seed, dev, dt), _randn((B, KV, S, D), seed + 1, dev, dt),
            _randn((B, KV, S, D), seed + 2, dev, dt))


def _decode_ref(q, k, v):
    B, H, D = q.shape
    KV = k.shape[1]
    kk = k.float().repeat_interleave(H // KV, 1)
    vv = v.float().repeat_interleave(H // KV, 1)
    s = torch.einsum("bhd,bhsd->bhs", q.float(), kk) / math.sqrt(D)
    return torch.einsum("bhs,bhsd->bhd", s.softmax(-1), vv)


def _decode_base(q, k, v):
    H, KV = q.shape[1], k.shape[1]
    return F.scaled_dot_product_attention(q.unsqueeze(2), k, v, enable_gqa=(H != KV)).squeeze(2)


def _mk_prefill(d, seed, dev, dt):
    B, H, KV, S, D = d["B"], d["H"], d["KV"], d["S"], d["D"]
    return (_randn((B, H, S, D), seed, dev, dt), _randn((B, KV, S, D), seed + 1, dev, dt),
            _randn((B, KV, S, D), seed + 2, dev, dt))


def _prefill_ref(q, k, v):
    H, KV = q.shape[1], k.shape[1]
    kk = k.float().repeat_interleave(H // KV, 1)
    vv = v.float().repeat_interleave(H // KV, 1)
    return F.scaled_dot_product_attention(q.float(), kk, vv, is_causal=True)


def _prefill_base(q, k, v):
    return F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=q.shape[1] != k.shape[1])


def _mk_rope(d, seed, dev, dt):
    S, B, H, D = d["S"], d["B"], d["H"], d["D"]
    x = _randn((B, S, H, D), seed, dev, dt)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
    f = torch.outer(torch.arange(S, device=dev, dtype=torch.float32), inv)
    return (x, f.cos(), f.sin())


def _rope_ref(x, cos, sin):
    d2 = x.shape[-1] // 2
    xf = x.float()
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat([xf[..., :d2] * c - xf[..., d2:] * s, xf[..., d2:] * c + xf[..., :d2] * s], -1)


def _mk_router(d, seed, dev, dt):
    return (_randn((d["M"], d["E"]), seed, dev, dt),)


def _topk_softmax_ref(logits, k=8):
    p = torch.softmax(logits.float(), -1)
    v, i = p.topk(k, -1)
    return torch.zeros_like(p).scatter(-1, i, v / v.sum(-1, keepdim=True))


def _mk_quant(d, seed, dev, dt):
    return (_randn((d["M"], d["N"]), seed, dev, dt, 3.0),)


def _quant_fp8_ref(x):
    xf = x.float()
    s = xf.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 448.0
    return (xf / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s


def _mk_ce(d, seed, dev, dt):
    g = _gen(seed + 5, dev)
    return (_randn((d["M"], d["N"]), seed, dev, dt, 2.0), torch.randint(0, d["N"], (d["M"],), generator=g, device=dev))


def _ce_ref(logits, tgt):
    return F.cross_entropy(logits.float(), tgt, reduction="none")


def _base_same_dtype(ref):
    return lambda *a: ref(*a)


SPECS: Dict[str, OpSpec] = {}


def _add(spec: OpSpec):
    SPECS[spec.name] = spec


_add(OpSpec("rmsnorm_bf16", "rmsnorm", "rmsnorm", _mk_rows, _rmsnorm_ref,
            lambda x, w: F.rms_norm(x, (x.shape[-1],), w, 1e-6),
            _rowwise("rmsnorm", "w = tl.load(W + cols, mask=m, other=0.0).to(tl.float32)\n    "
                     "r = 1.0 / tl.sqrt(tl.sum(x * x, 0) / N + eps)\n    y = x * r * w"),
            {"minimal": {"M": 64, "N": 512}, "primary": {"M": 4096, "N": 5120},
             "validation": [{"M": 8192, "N": 4096}, {"M": 333, "N": 2048}]}, "norm"))
_add(OpSpec("layernorm_bf16", "layernorm", "layernorm", _mk_rows, _layernorm_ref,
            lambda x, w: F.layer_norm(x, (x.shape[-1],), w, None, 1e-5),
            _rowwise("layernorm", "w = tl.load(W + cols, mask=m, other=0.0).to(tl.float32)\n    "
                     "mu = tl.sum(x, 0) / N\n    xc = tl.where(m, x - mu, 0.0)\n    "
                     "y = xc / tl.sqrt(tl.sum(xc * xc, 0) / N + eps) * w", 1e-5),
            {"minimal": {"M": 64, "N": 512}, "primary": {"M": 4096, "N": 4096},
             "validation": [{"M": 2048, "N": 8192}]}, "norm"))
_add(OpSpec("softmax_bf16", "softmax", "softmax", _mk_rows, _softmax_ref,
            lambda x, w: torch.softmax(x, -1),
            _rowwise("softmax", "x = tl.where(m, x, -float('inf'))\n    e = tl.exp(x - tl.max(x, 0))\n    "
                     "y = e / tl.sum(e, 0)"),
            {"minimal": {"M": 64, "N": 1024}, "primary": {"M": 4096, "N": 4096},
             "validation": [{"M": 1024, "N": 32000}]}, "reduce"))
_add(OpSpec("silu_mul_bf16", "silu_mul", "silu_mul", _mk_pair, _silu_mul_ref,
            lambda a, b: F.silu(a) * b,
            _elem("silu_mul", "y = a / (1.0 + tl.exp(-a)) * b"),
            {"minimal": {"M": 64, "N": 1024}, "primary": {"M": 8192, "N": 17408},
             "validation": [{"M": 4096, "N": 14336}]}, "elementwise"))
_add(OpSpec("gelu_tanh_bf16", "gelu", "gelu_tanh", _mk_pair, _gelu_tanh_ref,
            lambda a, b: F.gelu(a, approximate="tanh"),
            _elem("gelu_tanh", "t = 0.7978845608028654 * (a + 0.044715 * a * a * a)\n    "
                  "y = 0.5 * a * (1.0 + (2.0 / (1.0 + tl.exp(-2.0 * t)) - 1.0))"),
            {"minimal": {"M": 64, "N": 1024}, "primary": {"M": 8192, "N": 8192}, "validation": []}, "elementwise"))
_add(OpSpec("gemm_bf16", "gemm", "gemm", _mk_gemm, _gemm_ref, lambda a, b: a @ b.t(),
            _GEMM_SEED.replace("{entry}", "gemm"),
            {"minimal": {"M": 128, "N": 128, "K": 256}, "primary": {"M": 8192, "N": 5120, "K": 5120},
             "validation": [{"M": 4096, "N": 17408, "K": 5120}, {"M": 8192, "N": 5120, "K": 17408}]}, "gemm"))
_add(OpSpec("flash_attn_decode_bf16", "attention_decode", "decode_attention", _mk_decode, _decode_ref,
            _decode_base, _DECODE_SEED.replace("{entry}", "decode_attention"),
            {"minimal": {"B": 2, "H": 8, "KV": 2, "S": 256, "D": 128},
             "primary": {"B": 8, "H": 40, "KV": 8, "S": 4096, "D": 128},
             "validation": [{"B": 32, "H": 40, "KV": 8, "S": 1024, "D": 128}]}, "attention"))
_add(OpSpec("flash_attn_prefill_bf16", "attention_prefill", "prefill_attention", _mk_prefill, _prefill_ref,
            _prefill_base, "import torch\n\n\ndef prefill_attention(q, k, v):\n    raise NotImplementedError\n",
            {"minimal": {"B": 1, "H": 4, "KV": 1, "S": 256, "D": 128},
             "primary": {"B": 1, "H": 40, "KV": 8, "S": 4096, "D": 128}, "validation": []}, "attention"))
_add(OpSpec("rope_bf16", "rope", "rope", _mk_rope, _rope_ref, _rope_ref,
            "import torch\n\n\ndef rope(x, cos, sin):\n    d2 = x.shape[-1] // 2\n    c, s = cos[None, :, None, :], sin[None, :, None, :]\n"
            "    x1, x2 = x[..., :d2].float(), x[..., d2:].float()\n"
            "    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)\n",
            {"minimal": {"S": 64, "B": 1, "H": 4, "D": 128}, "primary": {"S": 8192, "B": 1, "H": 40, "D": 128},
             "validation": []}, "fusion"))
_add(OpSpec("topk_softmax_fp32", "topk_router", "topk_softmax", _mk_router, _topk_softmax_ref,
            _topk_softmax_ref,
            "import torch\n\n\ndef topk_softmax(logits, k=8):\n    p = torch.softmax(logits.float(), -1)\n"
            "    v, i = p.topk(k, -1)\n    return torch.zeros_like(p).scatter(-1, i, v / v.sum(-1, keepdim=True))\n",
            {"minimal": {"M": 64, "E": 128}, "primary": {"M": 16384, "E": 128}, "validation": []}, "moe", "fp32"))
_add(OpSpec("quant_fp8_pertoken", "quant", "quant_fp8", _mk_quant, _quant_fp8_ref, _quant_fp8_ref,
            "import torch\n\n\ndef quant_fp8(x):\n    xf = x.float()\n    s = xf.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 448.0\n"
            "    return (xf / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s\n",
            {"minimal": {"M": 64, "N": 1024}, "primary": {"M": 8192, "N": 5120}, "validation": []}, "quant", "fp8"))
_add(OpSpec("cross_entropy_bf16", "cross_entropy", "cross_entropy", _mk_ce, _ce_ref,
            lambda z, t: F.cross_entropy(z, t, reduction="none"),
            "import torch\n\n\ndef cross_entropy(logits, target):\n    z = logits.float()\n"
            "    return torch.logsumexp(z, -1) - z.gather(-1, target[:, None])[:, 0]\n",
            {"minimal": {"M": 16, "N": 32000}, "primary": {"M": 4096, "N": 151936}, "validation": []}, "reduce"))

# generated elementwise families (the reference's generic op generator, reduced)
_UNARY = {"relu": "tl.maximum(a, 0.0)", "sigmoid": "1.0 / (1.0 + tl.exp(-a))", "exp": "tl.exp(a)",
          "square": "a * a", "abs": "tl.abs(a)", "silu": "a / (1.0 + tl.exp(-a))"}
_UNARY_REF = {"relu": torch.relu, "sigmoid": torch.sigmoid, "exp": torch.exp, "square": torch.square,
              "abs": torch.abs, "silu": F.silu}
_BINARY = {"add": ("a + b", torch.add), "mul": ("a * b", torch.mul), "sub": ("a - b", torch.sub),
           "max": ("tl.maximum(a, b)", torch.maximum)}
for _n, _e in _UNARY.items():
    _r = _UNARY_REF[_n]
    _add(OpSpec(f"gen_{_n}_bf16", _n, _n, _mk_pair, (lambda r: lambda a, b: r(a.float()))(_r),
                (lambda r: lambda a, b: r(a))(_r), _elem(_n, f"y = {_e}"),
                {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 4096, "N": 4096}, "validation": []},
                "unary"))
for _n, (_e, _r) in _BINARY.items():
    _add(OpSpec(f"gen_{_n}_bf16", _n, _n, _mk_pair, (lambda r: lambda a, b: r(a.float(), b.float()))(_r),
                (lambda r: lambda a, b: r(a, b))(_r), _elem(_n, f"y = {_e}"),
                {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 4096, "N": 4096}, "validation": []},
                "binary"))


# generated breadth families (kore_b200.tasks.breadth)
def _register_breadth():
    from .breadth import build
    from .breadth_attn import build as build_attn
    from .breadth_ext import build as build_ext
    from .breadth_fx import build as build_fx
    from .breadth_train import build as build_train
    from .core_ext import build as build_core
    from .genops import build as build_gen
    for _s in build() + build_train() + build_ext() + build_fx() + build_attn():
        if _s.name not in SPECS:
            _add(_s)
    for _n, _s in list(build_gen().items()) + list(build_core().items()):
        if _n not in SPECS:          # the hand-written gen_* seeds above take precedence
            _add(_s)


_register_breadth()
