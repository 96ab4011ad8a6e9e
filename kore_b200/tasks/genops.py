"""The ``gen_*`` operator family: 67 generic operators x {bf16, fp16, fp32}.

Five classes, each with an fp32 PyTorch oracle, a vendor baseline on B200 and
a correct PyTorch seed the policy starts from:

* unary elementwise (24) and binary elementwise (8) over a flat tensor;
* row reductions [M, N] -> [M] (8);
* pointwise fusions of two or three inputs (16): the baseline is PyTorch eager,
  one kernel per op, so a single fused kernel has real headroom;
* GEMM with a fused bias / activation epilogue (11): the baseline is the
  cuBLAS matmul followed by separate epilogue kernels.

Task ids are ``gen_<op>_<dtype>`` and the operator names are those of the
reference's generic generator (kore/tasks/_genops.py:93-335), so datasets and
held-out lists keyed on them carry over; inputs, oracles and seeds are written
here from the operators' definitions. Positive-domain unary ops (sqrt, rsqrt,
reciprocal, log) and the divisor of ``div`` draw |randn| + 0.1.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch
import torch.nn.functional as F

from .spec import OpSpec, _randn

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
SNR = {"bf16": 30.0, "fp16": 30.0, "fp32": 40.0}

_G = "F.gelu({}, approximate='tanh')"

UNARY: Dict[str, Tuple[str, str]] = {   # name -> (expression of a, domain)
    "relu": ("torch.relu(a)", "signed"), "relu6": ("F.relu6(a)", "signed"),
    "leaky_relu": ("F.leaky_relu(a, 0.01)", "signed"), "silu": ("F.silu(a)", "signed"),
    "sigmoid": ("torch.sigmoid(a)", "signed"), "hardsigmoid": ("F.hardsigmoid(a)", "signed"),
    "tanh": ("torch.tanh(a)", "signed"), "hardtanh": ("F.hardtanh(a)", "signed"),
    "hardswish": ("F.hardswish(a)", "signed"), "softsign": ("F.softsign(a)", "signed"),
    "elu": ("F.elu(a)", "signed"), "softplus": ("F.softplus(a)", "signed"), "mish": ("F.mish(a)", "signed"),
    "gelu_tanh": (_G.format("a"), "signed"), "gelu_quick": ("a * torch.sigmoid(1.702 * a)", "signed"),
    "exp": ("torch.exp(a)", "signed"), "abs": ("torch.abs(a)", "signed"), "neg": ("torch.neg(a)", "signed"),
    "square": ("torch.square(a)", "signed"), "sign": ("torch.sign(a)", "signed"),
    "sqrt": ("torch.sqrt(a)", "pos"), "rsqrt": ("torch.rsqrt(a)", "pos"),
    "reciprocal": ("torch.reciprocal(a)", "pos"), "log": ("torch.log(a)", "pos"),
}
BINARY: Dict[str, Tuple[str, str]] = {  # name -> (expression of a, b; domain of b)
    "add": ("a + b", "signed"), "mul": ("a * b", "signed"), "sub": ("a - b", "signed"),
    "maximum": ("torch.maximum(a, b)", "signed"), "minimum": ("torch.minimum(a, b)", "signed"),
    "add_relu": ("torch.relu(a + b)", "signed"), "mul_sig": ("a * torch.sigmoid(b)", "signed"),
    "div": ("a / b", "pos"),
}
REDUCE: Dict[str, str] = {
    "row_sum": "x.sum(-1)", "row_mean": "x.mean(-1)", "row_max": "x.amax(-1)", "row_l2": "x.norm(p=2, dim=-1)",
    "row_rms": "x.pow(2).mean(-1).sqrt()", "row_l1": "x.abs().sum(-1)", "row_max_abs": "x.abs().amax(-1)",
    "row_min": "x.amin(-1)",
}
FUSION: Dict[str, Tuple[str, int]] = {   # name -> (expression, arity)
    "add_gelu": (_G.format("a + b"), 2), "add_silu": ("F.silu(a + b)", 2), "silu_mul": ("F.silu(a) * b", 2),
    "gelu_mul": (_G.format("a") + " * b", 2), "sigmoid_mul": ("torch.sigmoid(a) * b", 2),
    "mul_relu": ("torch.relu(a * b)", 2), "mul_tanh": ("torch.tanh(a * b)", 2), "fma": ("a * b + c", 3),
    "fma_relu": ("torch.relu(a * b + c)", 3), "fma_gelu": (_G.format("a * b + c"), 3),
    "add_add_relu": ("torch.relu(a + b + c)", 3), "add_mul": ("(a + b) * c", 3),
    "reglu": ("torch.relu(a) * b", 2), "sub_relu": ("torch.relu(a - b)", 2),
    "add_mul_relu": ("torch.relu((a + b) * c)", 3), "mul_add_tanh": ("torch.tanh(a * b + c)", 3),
}
ACTS = {"none": "y", "relu": "torch.relu(y)", "gelu": _G.format("y"), "silu": "F.silu(y)",
        "tanh": "torch.tanh(y)", "sigmoid": "torch.sigmoid(y)"}
GEMM_FUSION: Dict[str, Tuple[bool, str]] = {   # name -> (bias, activation)
    "gemm_bias": (True, "none"), "gemm_relu": (False, "relu"), "gemm_gelu": (False, "gelu"),
    "gemm_silu": (False, "silu"), "gemm_bias_relu": (True, "relu"), "gemm_bias_gelu": (True, "gelu"),
    "gemm_bias_silu": (True, "silu"), "gemm_tanh": (False, "tanh"), "gemm_sigmoid": (False, "sigmoid"),
    "gemm_bias_tanh": (True, "tanh"), "gemm_bias_sigmoid": (True, "sigmoid"),
}

_FLAT_SHAPES = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 8192},
                "validation": [{"M": 1, "N": 4097}, {"M": 4096, "N": 16384}]}
_ROW_SHAPES = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 8192},
               "validation": [{"M": 333, "N": 4097}, {"M": 65536, "N": 512}]}
_GEMM_SHAPES = {"minimal": {"M": 64, "N": 128, "K": 64}, "primary": {"M": 4096, "N": 4096, "K": 4096},
                "validation": [{"M": 8192, "N": 14336, "K": 4096}, {"M": 1, "N": 4096, "K": 4096},
                               {"M": 1000, "N": 1024, "K": 4096}]}


def _draw(shape, seed, dev, dt, domain):
    x = _randn(shape, seed, dev, torch.float32)
    if domain == "pos":
        x = x.abs() + 0.1
    return x.to(dt)


def _fn(args: str, expr: str):
    return eval(f"lambda {args}: {expr}", {"torch": torch, "F": F})


def _fp32(f):
    return lambda *x: f(*(t.float() if t.is_floating_point() else t for t in x))


def _seed(entry: str, args: str, expr: str) -> str:
    return (f"import torch\nimport torch.nn.functional as F\n\n\ndef {entry}({args}):\n"
            f"    return ({expr}).to({args.split(',')[0].strip()}.dtype)\n")


def _unary(name, expr, dom, dt) -> OpSpec:
    mk = lambda d, s, dev, t, dom=dom: (_draw((d["M"] * d["N"],), s, dev, t, dom),)
    f = _fn("a", expr)
    return OpSpec(f"gen_{name}_{dt}", f"elementwise_{name}", name, mk, _fp32(f), f, _seed(name, "a", expr),
                  _FLAT_SHAPES, "gen_unary", dt, SNR[dt])


def _binary(name, expr, dom_b, dt) -> OpSpec:
    def mk(d, s, dev, t, dom_b=dom_b):
        n = d["M"] * d["N"]
        return _draw((n,), s, dev, t, "signed"), _draw((n,), s + 11, dev, t, dom_b)
    f = _fn("a, b", expr)
    return OpSpec(f"gen_{name}_{dt}", f"elementwise_{name}", name, mk, _fp32(f), f, _seed(name, "a, b", expr),
                  _FLAT_SHAPES, "gen_binary", dt, SNR[dt])


def _reduce(name, expr, dt) -> OpSpec:
    mk = lambda d, s, dev, t: (_draw((d["M"], d["N"]), s, dev, t, "signed"),)
    f = _fn("x", expr)
    return OpSpec(f"gen_{name}_{dt}", f"reduce_{name}", name, mk, _fp32(f), f, _seed(name, "x", expr),
                  _ROW_SHAPES, "gen_reduce", dt, SNR[dt])


def _fusion(name, expr, arity, dt) -> OpSpec:
    args = "a, b" if arity == 2 else "a, b, c"
    mk = lambda d, s, dev, t, k=arity: tuple(_draw((d["M"], d["N"]), s + 5 * i, dev, t, "signed")
                                             for i in range(k))
    f = _fn(args, expr)
    return OpSpec(f"gen_{name}_{dt}", f"fusion_{name}", name, mk, _fp32(f), f, _seed(name, args, expr),
                  _ROW_SHAPES, "gen_fusion", dt, SNR[dt])


def _gemm_fusion(name, bias, act, dt) -> OpSpec:
    def mk(d, s, dev, t, bias=bias):
        a = _randn((d["M"], d["K"]), s, dev, t, 1.0)
        b = _randn((d["N"], d["K"]), s + 1, dev, t, d["K"] ** -0.5)
        out = (a, b)
        if bias:
            out += (_randn((d["N"],), s + 2, dev, t, 0.1),)
        return out
    args = "a, b, bias" if bias else "a, b"
    body = "a @ b.t()" + (" + bias" if bias else "")
    expr = ACTS[act].replace("y", f"({body})")
    f = _fn(args, expr)
    return OpSpec(f"gen_{name}_{dt}", "gemm", name, mk, _fp32(f), f, _seed(name, args, expr),
                  _GEMM_SHAPES, "gen_gemm_fusion", dt, SNR[dt])


def build() -> Dict[str, OpSpec]:
    out: Dict[str, OpSpec] = {}
    for dt in DTYPES:
        for n, (e, dom) in UNARY.items():
            out[f"gen_{n}_{dt}"] = _unary(n, e, dom, dt)
        for n, (e, dom) in BINARY.items():
            out[f"gen_{n}_{dt}"] = _binary(n, e, dom, dt)
        for n, e in REDUCE.items():
            out[f"gen_{n}_{dt}"] = _reduce(n, e, dt)
        for n, (e, k) in FUSION.items():
            out[f"gen_{n}_{dt}"] = _fusion(n, e, k, dt)
        for n, (b, a) in GEMM_FUSION.items():
            out[f"gen_{n}_{dt}"] = _gemm_fusion(n, b, a, dt)
    return out


def op_names():
    return sorted(set(UNARY) | set(BINARY) | set(REDUCE) | set(FUSION) | set(GEMM_FUSION))
