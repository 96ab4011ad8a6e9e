"""Breadth task families, generated programmatically (environment content).

Each family is a table of operations; every entry becomes one
:class:`~kore_b200.tasks.ops_library.OpSpec` per dtype (and per shape class
where the shape matters), with an fp32 PyTorch oracle, a vendor baseline
(the same op through PyTorch's CUDA kernels / cuBLAS / cuDNN in the task
dtype) and a correct PyTorch seed the policy starts from. Families:
unary, binary, gated activations, row reductions, normalisations (plain,
weighted, residual-fused, gated), GEMM + epilogue fusions over LLM shapes,
batched GEMM, decode / prefill / sliding-window / soft-capped attention,
MoE routing / permute / combine, training ops (cross-entropy fwd/bwd,
softmax and log-softmax backward, AdamW / Lion / SGD steps, grad-norm),
sampling (temperature, top-k, top-p, min-p, repetition penalty), scans and
linear recurrences, depthwise causal conv1d / conv2d / pooling,
quantisation (fp8 per-tensor / per-token / per-block, int8), sorting and
top-k, and RoPE variants.
Reference parity: the breadth engines and generic op generator of the
reference (kore/tasks/_genops.py:93-335 and the genb_* modules listed in
kore/tasks/breadth/: attn_ext, gemm_ext, moe_ext, norm_ext, reduce_ext,
sample_ext, ssm_ext, train_ops, fused_ext, conv, quant_ext, seq,
sort_sparse), written from the operation definitions, not from that code.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, List, Tuple

import torch
import torch.nn.functional as F

from .spec import OpSpec, _randn

DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}

_ROWS = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 4096, "N": 8192},
         "validation": [{"M": 333, "N": 4096}, {"M": 8192, "N": 2048}]}
_FLAT = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 8192}, "validation": [{"M": 1000, "N": 4097}]}


def _seed(entry: str, args: str, body: str) -> str:
    return f"import math\n\nimport torch\nimport torch.nn.functional as F\n\n\ndef {entry}({args}):\n    return {body}\n"


def _cast(dt):
    """The dtype candidates compute in (tasks with fp8 data use bf16 inputs)."""
    return DT.get(dt, torch.bfloat16)


# ------------------------------------------------------------------ inputs
def _mk_flat2(d, s, dev, dt):
    n = d["M"] * d["N"]
    return _randn((n,), s, dev, dt), _randn((n,), s + 7, dev, dt)


def _mk_rows1(d, s, dev, dt):
    return (_randn((d["M"], d["N"]), s, dev, dt),)


def _mk_rows_w(d, s, dev, dt):
    x = _randn((d["M"], d["N"]), s, dev, dt)
    w = (1 + 0.1 * _randn((d["N"],), s + 1, dev, torch.float32)).to(dt)
    r = _randn((d["M"], d["N"]), s + 2, dev, dt)
    b = (0.1 * _randn((d["N"],), s + 3, dev, torch.float32)).to(dt)
    return x, w, r, b


# ------------------------------------------------------------------ elementwise
UNARY: Dict[str, str] = {
    "relu": "torch.relu(a)", "relu6": "F.relu6(a)", "leaky_relu": "F.leaky_relu(a, 0.01)", "elu": "F.elu(a)",
    "selu": "F.selu(a)", "celu": "F.celu(a)", "gelu": "F.gelu(a)", "gelu_tanh": "F.gelu(a, approximate='tanh')",
    "silu": "F.silu(a)", "mish": "F.mish(a)", "softplus": "F.softplus(a)", "softsign": "F.softsign(a)",
    "tanh": "torch.tanh(a)", "sigmoid": "torch.sigmoid(a)", "hardsigmoid": "F.hardsigmoid(a)",
    "hardswish": "F.hardswish(a)", "hardtanh": "F.hardtanh(a)", "logsigmoid": "F.logsigmoid(a)",
    "tanhshrink": "F.tanhshrink(a)", "softshrink": "F.softshrink(a, 0.5)", "hardshrink": "F.hardshrink(a, 0.5)",
    "exp_clamped": "torch.exp(a.clamp(max=10.0))", "exp2_clamped": "torch.exp2(a.clamp(max=10.0))",
    "expm1_clamped": "torch.expm1(a.clamp(max=10.0))", "log1p_abs": "torch.log1p(a.abs())",
    "log_abs": "torch.log(a.abs() + 1e-3)", "sqrt_abs": "torch.sqrt(a.abs())",
    "rsqrt_abs": "torch.rsqrt(a.abs() + 1e-2)", "reciprocal_safe": "1.0 / (a.abs() + 0.5)",
    "square": "a * a", "cube": "a * a * a", "abs": "a.abs()", "neg": "-a", "sign": "torch.sign(a)",
    "floor": "torch.floor(a * 4)", "ceil": "torch.ceil(a * 4)", "round": "torch.round(a * 4)",
    "sin": "torch.sin(a)", "cos": "torch.cos(a)", "erf": "torch.erf(a)", "erfc": "torch.erfc(a)",
    "clamp": "a.clamp(-0.5, 0.5)", "quick_gelu": "a * torch.sigmoid(1.702 * a)",
    "squareplus": "0.5 * (a + torch.sqrt(a * a + 4.0))", "swish_beta": "a * torch.sigmoid(1.5 * a)",
}

BINARY: Dict[str, str] = {
    "add": "a + b", "sub": "a - b", "mul": "a * b", "div_safe": "a / (b.abs() + 0.5)", "maximum": "torch.maximum(a, b)",
    "minimum": "torch.minimum(a, b)", "pow_abs": "a.abs().clamp(min=1e-3) ** b.clamp(-2.0, 2.0)",
    "atan2": "torch.atan2(a, b)", "hypot": "torch.hypot(a, b)", "lerp": "torch.lerp(a, b, 0.3)",
    "squared_diff": "(a - b) ** 2", "abs_diff": "(a - b).abs()",
    "bce_logits": "F.softplus(a) - a * torch.sigmoid(b)", "add_relu": "torch.relu(a + b)",
    "mul_add": "a * b + a", "where_gt": "torch.where(a > b, a, b * 0.5)",
    "silu_mul": "F.silu(a) * b", "gelu_mul": "F.gelu(a, approximate='tanh') * b", "relu_mul": "torch.relu(a) * b",
    "sigmoid_mul": "torch.sigmoid(a) * b", "relu2_mul": "torch.relu(a) ** 2 * b", "scaled_add": "0.7 * a + 1.3 * b",
}


def _ew_spec(kind: str, name: str, expr: str, dt: str) -> OpSpec:
    entry = name
    if kind == "unary":
        mk = lambda d, s, dev, t: (_mk_flat2(d, s, dev, t)[0],)
        args = "a"
    else:
        mk = _mk_flat2
        args = "a, b"
    f = eval(f"lambda {args}: {expr}", {"torch": torch, "F": F, "math": math})
    ref = (lambda f: (lambda *x: f(*(t.float() for t in x))))(f)
    op = name if any(k in name for k in ("relu", "gelu", "silu")) else f"elementwise_{name}"
    return OpSpec(f"genb_{kind}_{name}_{dt}", op, entry, mk, ref, f, _seed(entry, args, expr), _FLAT,
                  kind, dt)


# ------------------------------------------------------------------ reductions / norms
REDUCE: Dict[str, str] = {
    "row_sum": "x.sum(-1)", "row_mean": "x.mean(-1)", "row_max": "x.amax(-1)", "row_min": "x.amin(-1)",
    "row_absmax": "x.abs().amax(-1)", "row_l2norm": "x.norm(dim=-1)", "row_var": "x.var(-1, unbiased=False)",
    "row_std": "x.std(-1, unbiased=False)", "logsumexp": "torch.logsumexp(x, -1)", "softmax": "torch.softmax(x, -1)",
    "log_softmax": "torch.log_softmax(x, -1)", "softmax_temp": "torch.softmax(x / 0.7, -1)",
    "entropy": "-(torch.softmax(x, -1) * torch.log_softmax(x, -1)).sum(-1)",
    "l2_normalize": "F.normalize(x, dim=-1)", "cumsum": "torch.cumsum(x, -1)",
    "cummax": "torch.cummax(x, -1).values", "argmax_onehot": "F.one_hot(x.argmax(-1), x.shape[-1]).to(x.dtype)",
    "rmsnorm_plain": "x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)",
    "layernorm_plain": "F.layer_norm(x, (x.shape[-1],))",
}

NORMS: Dict[str, str] = {
    "rmsnorm_w": "x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w",
    "add_rmsnorm": "(x + r) * torch.rsqrt((x + r).pow(2).mean(-1, keepdim=True) + 1e-6) * w",
    "layernorm_wb": "F.layer_norm(x, (x.shape[-1],), w, b, 1e-5)",
    "add_layernorm": "F.layer_norm(x + r, (x.shape[-1],), w, b, 1e-5)",
    "rmsnorm_gated": "x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w * F.silu(r)",
    "rmsnorm_one_plus_w": "x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w)",
    "rmsnorm_bias": "x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w + b",
    "add_rmsnorm_residual_out": "torch.cat([(x + r) * torch.rsqrt((x + r).pow(2).mean(-1, keepdim=True) + 1e-6) * w, x + r], -1)",
    "scale_shift_norm": "F.layer_norm(x, (x.shape[-1],)) * (1 + w) + b",
    "groupnorm8": "F.group_norm(x, 8, w, b)",
}


def _row_spec(kind: str, name: str, expr: str, dt: str, with_w: bool) -> OpSpec:
    args = "x, w, r, b" if with_w else "x"
    f = eval(f"lambda {args}: {expr}", {"torch": torch, "F": F})
    ref = (lambda f: (lambda *x: f(*(t.float() for t in x))))(f)
    mk = _mk_rows_w if with_w else _mk_rows1
    op = {"row_sum": "reduce", "softmax": "softmax", "log_softmax": "log_softmax"}.get(name, name)
    if "rmsnorm" in name:
        op = "fused_add_rmsnorm" if "add" in name else "rmsnorm"
    elif "layernorm" in name or "norm" in name:
        op = "layernorm"
    return OpSpec(f"genb_{kind}_{name}_{dt}", op, name, mk, ref, f, _seed(name, args, expr), _ROWS, kind, dt)


# ------------------------------------------------------------------ GEMM fusions
GEMM_EPI: Dict[str, str] = {
    "none": "y", "bias": "y + bias", "relu": "torch.relu(y + bias)", "gelu": "F.gelu(y + bias, approximate='tanh')",
    "silu": "F.silu(y + bias)", "sigmoid": "torch.sigmoid(y)", "tanh": "torch.tanh(y)", "residual": "y + res",
    "scale_residual": "0.5 * y + res", "relu2": "torch.relu(y) ** 2",
}
GEMM_SHAPES: Dict[str, Dict[str, int]] = {
    "square4k": {"M": 4096, "N": 4096, "K": 4096}, "qkv14b": {"M": 8192, "N": 7168, "K": 5120},
    "up14b": {"M": 8192, "N": 17408, "K": 5120}, "down14b": {"M": 8192, "N": 5120, "K": 17408},
    "decode14b": {"M": 16, "N": 5120, "K": 5120},
}


def _mk_gemm_epi(d, s, dev, dt):
    a = _randn((d["M"], d["K"]), s, dev, dt, 1.0 / math.sqrt(d["K"]) ** 0.5)
    b = _randn((d["N"], d["K"]), s + 1, dev, dt, 1.0 / math.sqrt(d["K"]) ** 0.5)
    bias = _randn((d["N"],), s + 2, dev, dt, 0.1)
    res = _randn((d["M"], d["N"]), s + 3, dev, dt)
    return a, b, bias, res


def _gemm_spec(epi: str, shape: str, dt: str) -> OpSpec:
    expr = GEMM_EPI[epi]
    body = f"(lambda y: {expr})(a @ b.t())"
    f = eval(f"lambda a, b, bias, res: {body}", {"torch": torch, "F": F})
    ref = (lambda f: (lambda *x: f(*(t.float() for t in x))))(f)
    d = GEMM_SHAPES[shape]
    shapes = {"minimal": {"M": 128, "N": 128, "K": 256}, "primary": dict(d), "validation": []}
    name = f"gemm_{epi}"
    return OpSpec(f"genb_gemm_{epi}_{shape}_{dt}", "gemm", name, _mk_gemm_epi, ref, f,
                  _seed(name, "a, b, bias, res", body), shapes, "gemm_fusion", dt)


def _mk_bmm(d, s, dev, dt):
    return (_randn((d["B"], d["M"], d["K"]), s, dev, dt, 0.1), _randn((d["B"], d["K"], d["N"]), s + 1, dev, dt, 0.1))


BMM_SHAPES = {"heads32_s512": {"B": 32, "M": 512, "N": 512, "K": 128},
              "heads64_s2k": {"B": 64, "M": 2048, "N": 128, "K": 2048},
              "experts8": {"B": 8, "M": 2048, "N": 768, "K": 2048}}


# ------------------------------------------------------------------ attention
def _mk_attn(d, s, dev, dt):
    B, H, KV, S, D = d["B"], d["H"], d["KV"], d["S"], d["D"]
    Sq = d.get("Sq", S)
    return (_randn((B, H, Sq, D), s, dev, dt), _randn((B, KV, S, D), s + 1, dev, dt),
            _randn((B, KV, S, D), s + 2, dev, dt))


def _attn_fn(causal: bool, window: int = 0, softcap: float = 0.0):
    def f(q, k, v):
        H, KV = q.shape[1], k.shape[1]
        if H != KV:
            k = k.repeat_interleave(H // KV, 1)
            v = v.repeat_interleave(H // KV, 1)
        sc = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
        if softcap:
            sc = softcap * torch.tanh(sc / softcap)
        Sq, S = q.shape[2], k.shape[2]
        qi = torch.arange(Sq, device=q.device)[:, None] + (S - Sq)
        ki = torch.arange(S, device=q.device)[None, :]
        mask = torch.zeros(Sq, S, dtype=torch.bool, device=q.device)
        if causal:
            mask |= ki > qi
        if window:
            mask |= ki <= qi - window
        sc = sc.masked_fill(mask, float("-inf"))
        return torch.softmax(sc.float(), -1).to(v.dtype) @ v
    return f


def _attn_base(causal: bool, window: int = 0, softcap: float = 0.0):
    plain = _attn_fn(causal, window, softcap)

    def f(q, k, v):
        if window or softcap or q.shape[2] != k.shape[2] and causal:
            return plain(q, k, v)
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal and q.shape[2] > 1, enable_gqa=True)
    return f


ATTN: List[Tuple[str, str, Dict[str, int], bool, int, float]] = []
for (h, kv) in ((32, 8), (40, 8), (64, 8), (32, 32), (32, 1), (16, 2)):
    for (b, sk) in ((8, 4096), (32, 1024), (1, 16384)):
        ATTN.append((f"decode_h{h}kv{kv}_b{b}_s{sk}", "attention_decode",
                     {"B": b, "H": h, "KV": kv, "S": sk, "Sq": 1, "D": 128}, False, 0, 0.0))
for (h, kv) in ((32, 8), (40, 8), (16, 16)):
    for sq in (1024, 4096):
        for causal in (True, False):
            ATTN.append((f"prefill_{'causal' if causal else 'full'}_h{h}kv{kv}_s{sq}", "attention_prefill",
                         {"B": 1, "H": h, "KV": kv, "S": sq, "D": 128}, causal, 0, 0.0))
ATTN += [("prefill_sliding1k_h32kv8_s4096", "attention_prefill", {"B": 1, "H": 32, "KV": 8, "S": 4096, "D": 128},
          True, 1024, 0.0),
         ("prefill_sliding4k_h32kv8_s8192", "attention_prefill", {"B": 1, "H": 32, "KV": 8, "S": 8192, "D": 128},
          True, 4096, 0.0),
         ("prefill_softcap30_h16kv8_s2048", "attention_prefill", {"B": 1, "H": 16, "KV": 8, "S": 2048, "D": 128},
          True, 0, 30.0),
         ("chunked_prefill_h32kv8_q512_kv4096", "attention_prefill",
          {"B": 2, "H": 32, "KV": 8, "S": 4096, "Sq": 512, "D": 128}, True, 0, 0.0),
         ("prefill_hd64_h16kv4_s2048", "attention_prefill", {"B": 2, "H": 16, "KV": 4, "S": 2048, "D": 64},
          True, 0, 0.0)]


# ------------------------------------------------------------------ MoE
def _mk_router(d, s, dev, dt):
    return (_randn((d["M"], d["E"]), s, dev, dt),)


def _topk_softmax(k, renorm=True, sigmoid=False):
    def f(z):
        p = torch.sigmoid(z) if sigmoid else torch.softmax(z, -1)
        v, i = p.topk(k, -1)
        if renorm:
            v = v / v.sum(-1, keepdim=True)
        return torch.zeros_like(p).scatter(-1, i, v)
    return f


def _mk_permute(d, s, dev, dt):
    x = _randn((d["M"], d["D"]), s, dev, dt)
    g = torch.Generator(device=dev)
    g.manual_seed(s)
    idx = torch.randint(0, d["M"], (d["M"] * d["K"],), generator=g, device=dev)
    return x, idx


def _mk_combine(d, s, dev, dt):
    y = _randn((d["M"] * d["K"], d["D"]), s, dev, dt)
    w = torch.softmax(_randn((d["M"], d["K"]), s + 1, dev, torch.float32), -1).to(dt)
    return y, w


# ------------------------------------------------------------------ training ops
def _mk_ce(d, s, dev, dt):
    z = _randn((d["M"], d["N"]), s, dev, dt, 2.0)
    g = torch.Generator(device=dev)
    g.manual_seed(s)
    return z, torch.randint(0, d["N"], (d["M"],), generator=g, device=dev)


def _ce_bwd(z, t):
    p = torch.softmax(z.float(), -1)
    return p - F.one_hot(t, z.shape[-1]).float()


def _mk_grad_pair(d, s, dev, dt):
    return _randn((d["M"], d["N"]), s, dev, dt), _randn((d["M"], d["N"]), s + 1, dev, dt)


def _softmax_bwd(x, g):
    y = torch.softmax(x.float(), -1)
    return y * (g.float() - (g.float() * y).sum(-1, keepdim=True))


def _logsoftmax_bwd(x, g):
    return g.float() - torch.softmax(x.float(), -1) * g.float().sum(-1, keepdim=True)


def _mk_opt(d, s, dev, dt):
    n = d["N"]
    p = _randn((n,), s, dev, torch.float32)
    g = _randn((n,), s + 1, dev, dt, 0.01)
    m = _randn((n,), s + 2, dev, torch.float32, 0.001)
    v = _randn((n,), s + 3, dev, torch.float32, 0.001).abs()
    return p, g, m, v


def _adamw(p, g, m, v, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, step=10):
    g = g.float()
    m2 = b1 * m + (1 - b1) * g
    v2 = b2 * v + (1 - b2) * g * g
    upd = (m2 / (1 - b1 ** step)) / ((v2 / (1 - b2 ** step)).sqrt() + eps)
    return torch.cat([p * (1 - lr * wd) - lr * upd, m2, v2])


def _lion(p, g, m, v, lr=1e-4, b1=0.9, b2=0.99, wd=0.01):
    g = g.float()
    c = torch.sign(b1 * m + (1 - b1) * g)
    return torch.cat([p * (1 - lr * wd) - lr * c, b2 * m + (1 - b2) * g])


def _sgd_mom(p, g, m, v, lr=1e-2, mu=0.9):
    m2 = mu * m + g.float()
    return torch.cat([p - lr * m2, m2])


def _grad_norm_clip(p, g, m, v, max_norm=1.0):
    gf = g.float()
    n = gf.norm()
    return gf * torch.clamp(max_norm / (n + 1e-6), max=1.0)


# ------------------------------------------------------------------ sampling
def _mk_logits(d, s, dev, dt):
    return (_randn((d["M"], d["N"]), s, dev, dt, 3.0),)


def _temperature_softmax(z, t=0.7):
    return torch.softmax(z.float() / t, -1)


def _greedy_onehot(z):
    return F.one_hot(z.argmax(-1), z.shape[-1]).float()


def _topk_mask(z, k=50):
    v, _ = z.topk(k, -1)
    return z.masked_fill(z < v[:, -1:], float("-inf"))


def _topp_mask(z, p=0.9):
    sp, si = torch.softmax(z.float(), -1).sort(-1, descending=True)
    keep_sorted = (sp.cumsum(-1) - sp) < p
    keep = torch.zeros_like(keep_sorted).scatter(-1, si, keep_sorted)
    return z.masked_fill(~keep, float("-inf"))


def _minp_mask(z, p=0.05):
    pr = torch.softmax(z.float(), -1)
    return z.masked_fill(pr < p * pr.amax(-1, keepdim=True), float("-inf"))


def _rep_penalty(z, pen=1.2):
    seen = torch.zeros_like(z, dtype=torch.bool)
    seen[:, ::7] = True
    return torch.where(seen, torch.where(z > 0, z / pen, z * pen), z)


# ------------------------------------------------------------------ scans / conv / quant / sort / rope
def _mk_scan(d, s, dev, dt):
    a = torch.sigmoid(_randn((d["B"], d["L"], d["D"]), s, dev, torch.float32)).to(dt)
    x = _randn((d["B"], d["L"], d["D"]), s + 1, dev, dt)
    return a, x


def _linear_recurrence(a, x):
    h = torch.zeros_like(x[:, 0])
    out = []
    for t in range(x.shape[1]):
        h = a[:, t] * h + x[:, t]
        out.append(h)
    return torch.stack(out, 1)


def _mk_conv1d(d, s, dev, dt):
    return _randn((d["B"], d["C"], d["L"]), s, dev, dt), _randn((d["C"], 1, d["W"]), s + 1, dev, dt, 0.5)


def _causal_dwconv(x, w):
    return F.conv1d(F.pad(x, (w.shape[-1] - 1, 0)), w, groups=x.shape[1])


def _mk_img(d, s, dev, dt):
    return _randn((d["B"], d["C"], d["H"], d["W"]), s, dev, dt), _randn((d["C"], d["C"], 3, 3), s + 1, dev, dt, 0.05)


def _fp8_per_tensor(x):
    xf = x.float()
    s = xf.abs().amax().clamp_min(1e-12) / 448.0
    return (xf / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s


def _fp8_per_block(x, blk=128):
    M, N = x.shape
    xb = x.float().reshape(M, N // blk, blk)
    s = xb.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 448.0
    return ((xb / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s).reshape(M, N)


def _int8_per_token(x):
    xf = x.float()
    s = xf.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 127.0
    return torch.round(xf / s).clamp(-127, 127) * s


def _mk_rope(d, s, dev, dt):
    S, H, D = d["S"], d["H"], d["D"]
    x = _randn((S, H, D), s, dev, dt)
    pos = torch.arange(S, device=dev, dtype=torch.float32)
    rot = d.get("R", D)
    inv = 1.0 / (1e6 ** (torch.arange(0, rot, 2, device=dev, dtype=torch.float32) / rot))
    ang = pos[:, None] * inv[None]
    return x, torch.cos(ang), torch.sin(ang)


def _rope_neox(x, cos, sin):
    r = cos.shape[-1] * 2
    xr, xp = x[..., :r].float(), x[..., r:].float()
    x1, x2 = xr[..., : r // 2], xr[..., r // 2:]
    c, s_ = cos[:, None], sin[:, None]
    return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_, xp], -1)


def _rope_gptj(x, cos, sin):
    xf = x.float()
    x1, x2 = xf[..., 0::2], xf[..., 1::2]
    c, s_ = cos[:, None], sin[:, None]
    return torch.stack([x1 * c - x2 * s_, x2 * c + x1 * s_], -1).flatten(-2)


# ------------------------------------------------------------------ assembly
def _fp32_of(f):
    return lambda *x: f(*(t.float() if t.is_floating_point() else t for t in x))


def build() -> List[OpSpec]:
    out: List[OpSpec] = []
    for dt in ("bf16", "fp16", "fp32"):
        out += [_ew_spec("unary", n, e, dt) for n, e in UNARY.items()]
        out += [_ew_spec("binary", n, e, dt) for n, e in BINARY.items()]
        out += [_row_spec("reduce", n, e, dt, False) for n, e in REDUCE.items()]
    for dt in ("bf16", "fp16"):
        out += [_row_spec("norm", n, e, dt, True) for n, e in NORMS.items()]
        out += [_gemm_spec(e, sh, dt) for e in GEMM_EPI for sh in GEMM_SHAPES]
        for nm, d in BMM_SHAPES.items():
            out.append(OpSpec(f"genb_bmm_{nm}_{dt}", "batched_gemm", "bmm", _mk_bmm, _fp32_of(torch.bmm), torch.bmm,
                              _seed("bmm", "a, b", "torch.bmm(a, b)"),
                              {"minimal": {"B": 2, "M": 64, "N": 64, "K": 64}, "primary": d, "validation": []},
                              "gemm_ext", dt))
    for name, op, d, causal, window, cap in ATTN:
        f = _attn_fn(causal, window, cap)
        mini = dict(d, B=1, S=min(d["S"], 256), **({"Sq": 1} if d.get("Sq") == 1 else {}))
        if "Sq" in mini and mini["Sq"] > 1:
            mini["Sq"] = min(mini["Sq"], 128)
        out.append(OpSpec(f"genb_attn_{name}_bf16", op, "attention", _mk_attn, _fp32_of(f),
                          _attn_base(causal, window, cap),
                          "import math\n\nimport torch\n\n\n" + _attn_seed(causal, window, cap),
                          {"minimal": mini, "primary": d, "validation": []}, "attention", "bf16"))
    for E, k in ((64, 2), (128, 8), (256, 8), (32, 4)):
        sh = {"minimal": {"M": 16, "E": E}, "primary": {"M": 16384, "E": E}, "validation": []}
        out.append(OpSpec(f"genb_moe_topk_softmax_e{E}k{k}_fp32", "topk_router", "router", _mk_router,
                          _topk_softmax(k), _topk_softmax(k), _router_seed(k, False), sh, "moe", "fp32"))
        out.append(OpSpec(f"genb_moe_topk_sigmoid_e{E}k{k}_fp32", "topk_router", "router", _mk_router,
                          _topk_softmax(k, sigmoid=True), _topk_softmax(k, sigmoid=True), _router_seed(k, True), sh,
                          "moe", "fp32"))
    for D, K in ((2048, 8), (5120, 2), (4096, 4)):
        sh = {"minimal": {"M": 16, "D": D, "K": K}, "primary": {"M": 8192, "D": D, "K": K}, "validation": []}
        out.append(OpSpec(f"genb_moe_permute_d{D}k{K}_bf16", "moe_permute", "permute", _mk_permute,
                          lambda x, i: x.float()[i], lambda x, i: x[i], _seed("permute", "x, idx", "x[idx]"), sh,
                          "moe", "bf16"))
        comb = lambda y, w: (y.float().view(w.shape[0], w.shape[1], -1) * w.float()[..., None]).sum(1)
        out.append(OpSpec(f"genb_moe_combine_d{D}k{K}_bf16", "moe_combine", "combine", _mk_combine, comb,
                          lambda y, w: (y.view(w.shape[0], w.shape[1], -1) * w[..., None]).sum(1),
                          _seed("combine", "y, w", "(y.float().view(w.shape[0], w.shape[1], -1) * w.float()[..., None]).sum(1)"),
                          sh, "moe", "bf16"))
    for V in (32000, 151936):
        sh = {"minimal": {"M": 8, "N": V}, "primary": {"M": 4096, "N": V}, "validation": []}
        out.append(OpSpec(f"genb_train_ce_fwd_v{V}_bf16", "cross_entropy", "ce", _mk_ce,
                          lambda z, t: F.cross_entropy(z.float(), t, reduction="none"),
                          lambda z, t: F.cross_entropy(z, t, reduction="none"),
                          _seed("ce", "z, t", "F.cross_entropy(z.float(), t, reduction='none')"), sh, "train", "bf16"))
        out.append(OpSpec(f"genb_train_ce_bwd_v{V}_bf16", "cross_entropy", "ce_bwd", _mk_ce, _ce_bwd, _ce_bwd,
                          _seed("ce_bwd", "z, t", "torch.softmax(z.float(), -1) - F.one_hot(t, z.shape[-1]).float()"),
                          sh, "train", "bf16"))
        for nm, fn, body in (("softmax_bwd", _softmax_bwd, "(lambda y: y * (g.float() - (g.float() * y).sum(-1, keepdim=True)))(torch.softmax(x.float(), -1))"),
                             ("logsoftmax_bwd", _logsoftmax_bwd, "g.float() - torch.softmax(x.float(), -1) * g.float().sum(-1, keepdim=True)")):
            out.append(OpSpec(f"genb_train_{nm}_v{V}_bf16", "log_softmax", nm, _mk_grad_pair, fn, fn,
                              _seed(nm, "x, g", body), sh, "train", "bf16"))
    for nm, fn in (("adamw", _adamw), ("lion", _lion), ("sgd_momentum", _sgd_mom), ("grad_norm_clip", _grad_norm_clip)):
        for n in (1 << 24, 14 << 20):
            sh = {"minimal": {"N": 4096}, "primary": {"N": n}, "validation": []}
            out.append(OpSpec(f"genb_train_{nm}_n{n >> 20}m_bf16", "optimizer", nm, _mk_opt, fn, fn,
                              _lib_seed(nm, "p, g, m, v", fn), sh, "train", "bf16"))
    for V in (32000, 151936):
        sh = {"minimal": {"M": 4, "N": V}, "primary": {"M": 256, "N": V}, "validation": []}
        for nm, fn in (("temperature_softmax", _temperature_softmax), ("topk_mask", _topk_mask),
                       ("topp_mask", _topp_mask), ("minp_mask", _minp_mask), ("repetition_penalty", _rep_penalty),
                       ("greedy_onehot", _greedy_onehot)):
            out.append(OpSpec(f"genb_sample_{nm}_v{V}_fp32", "softmax", nm, _mk_logits, _fp32_of(fn), fn,
                              _lib_seed(nm, "z", fn), sh, "sample", "fp32"))
    for (B, L, D) in ((4, 1024, 1024), (1, 4096, 2048)):
        sh = {"minimal": {"B": 1, "L": 64, "D": 64}, "primary": {"B": B, "L": L, "D": D}, "validation": []}
        out.append(OpSpec(f"genb_ssm_linear_recurrence_b{B}l{L}d{D}_fp32", "scan", "recurrence", _mk_scan,
                          _fp32_of(_linear_recurrence), _linear_recurrence, _lib_seed("recurrence", "a, x", _linear_recurrence),
                          sh, "ssm", "fp32"))
        out.append(OpSpec(f"genb_seq_cumsum_b{B}l{L}d{D}_fp32", "scan", "cumsum", _mk_scan,
                          lambda a, x: torch.cumsum(x.float(), 1), lambda a, x: torch.cumsum(x, 1),
                          _seed("cumsum", "a, x", "torch.cumsum(x.float(), 1)"), sh, "seq", "fp32"))
        out.append(OpSpec(f"genb_seq_cumprod_decay_b{B}l{L}d{D}_fp32", "scan", "cumprod", _mk_scan,
                          lambda a, x: torch.cumprod(a.float(), 1), lambda a, x: torch.cumprod(a, 1),
                          _seed("cumprod", "a, x", "torch.cumprod(a.float(), 1)"), sh, "seq", "fp32"))
    for (B, C, L, W) in ((8, 2048, 4096, 4), (4, 4096, 2048, 4)):
        sh = {"minimal": {"B": 1, "C": 64, "L": 128, "W": W}, "primary": {"B": B, "C": C, "L": L, "W": W}, "validation": []}
        out.append(OpSpec(f"genb_conv_causal_dwconv1d_c{C}l{L}_bf16", "conv", "dwconv", _mk_conv1d,
                          _fp32_of(_causal_dwconv), _causal_dwconv, _lib_seed("dwconv", "x, w", _causal_dwconv),
                          sh, "conv", "bf16"))
    for (B, C, H) in ((8, 64, 128), (16, 128, 56)):
        sh = {"minimal": {"B": 1, "C": 8, "H": 16, "W": 16}, "primary": {"B": B, "C": C, "H": H, "W": H}, "validation": []}
        out.append(OpSpec(f"genb_conv_conv2d3x3_c{C}h{H}_bf16", "conv", "conv2d", _mk_img,
                          lambda x, w: F.conv2d(x.float(), w.float(), padding=1), lambda x, w: F.conv2d(x, w, padding=1),
                          _seed("conv2d", "x, w", "F.conv2d(x.float(), w.float(), padding=1)"), sh, "conv", "bf16"))
        out.append(OpSpec(f"genb_conv_maxpool2d_c{C}h{H}_bf16", "conv", "maxpool", _mk_img,
                          lambda x, w: F.max_pool2d(x.float(), 2), lambda x, w: F.max_pool2d(x, 2),
                          _seed("maxpool", "x, w", "F.max_pool2d(x.float(), 2)"), sh, "conv", "bf16"))
        out.append(OpSpec(f"genb_conv_avgpool2d_c{C}h{H}_bf16", "conv", "avgpool", _mk_img,
                          lambda x, w: F.avg_pool2d(x.float(), 2), lambda x, w: F.avg_pool2d(x, 2),
                          _seed("avgpool", "x, w", "F.avg_pool2d(x.float(), 2)"), sh, "conv", "bf16"))
    qsh = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 5120}, "validation": []}
    for nm, fn in (("fp8_per_tensor", _fp8_per_tensor), ("fp8_per_block128", _fp8_per_block),
                   ("int8_per_token", _int8_per_token)):
        out.append(OpSpec(f"genb_quant_{nm}_bf16", "quant", "quant", _mk_rows1, _fp32_of(fn), fn,
                          _lib_seed("quant", "x", fn), qsh, "quant", "fp8" if "fp8" in nm else "bf16"))
    ssh = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 4096}, "validation": []}
    for nm, body in (("topk8_values", "x.float().topk(8, -1).values"), ("topk64_values", "x.float().topk(64, -1).values"),
                     ("sort_rows", "x.float().sort(-1).values"), ("sort_rows_desc", "x.float().sort(-1, descending=True).values"),
                     ("sparsify_2of4", "(lambda v: v * (v.abs() >= v.abs().topk(2, -1).values[..., -1:]))(x.float().view(x.shape[0], -1, 4)).view(x.shape)")):
        f = eval(f"lambda x: {body}", {"torch": torch})
        out.append(OpSpec(f"genb_sort_{nm}_bf16", "sort", nm, _mk_rows1, f, f, _seed(nm, "x", body), ssh,
                          "sort_sparse", "bf16"))
    for nm, fn, R in (("neox_full", _rope_neox, 128), ("neox_partial64", _rope_neox, 64), ("gptj", _rope_gptj, 128)):
        for H in (32, 40):
            sh = {"minimal": {"S": 16, "H": 4, "D": 128, "R": R}, "primary": {"S": 8192, "H": H, "D": 128, "R": R},
                  "validation": []}
            out.append(OpSpec(f"genb_rope_{nm}_h{H}_bf16", "rope", "rope", _mk_rope, _fp32_of(fn), fn,
                              _lib_seed("rope", "x, cos, sin", fn), sh, "fusion", "bf16"))
    return out


def _lib_seed(entry: str, args: str, fn: Callable) -> str:
    """A correct seed that calls the module-level PyTorch definition."""
    assert fn.__name__ != "<lambda>", entry
    return (f"from kore_b200.tasks.breadth import {fn.__name__} as _ref\n\n\n"
            f"def {entry}({args}):\n    return _ref({args})\n")


def _router_seed(k: int, sigmoid: bool) -> str:
    p = "torch.sigmoid(z.float())" if sigmoid else "torch.softmax(z.float(), -1)"
    return (f"import torch\n\n\ndef router(z):\n    p = {p}\n    v, i = p.topk({k}, -1)\n"
            f"    return torch.zeros_like(p).scatter(-1, i, v / v.sum(-1, keepdim=True))\n")


def _attn_seed(causal: bool, window: int, cap: float) -> str:
    return (f"from kore_b200.tasks.breadth import _attn_fn\n\n_F = _attn_fn({causal}, {window}, {cap})\n\n\n"
            "def attention(q, k, v):\n    return _F(q, k, v)\n")
