"""A typed composition grammar over torch primitives: the oracle builder of
minted tasks.

Values have one of two types: ``MAT`` (an ``[M, N]`` matrix) or ``ROW`` (an
``[M]`` vector, terminal: nothing follows a row reduction). A
:class:`Pipeline` is a source (``x``, an ``[M, K]`` input) followed by
stages; each :class:`Primitive` declares what it consumes and produces and
which auxiliary tensors it samples (a GEMM weight, a bias, a residual, a norm
scale). ``typecheck`` is the soundness gate; a well-typed pipeline *is* a
pure torch function, and that function (evaluated in fp32, cast to the task
dtype) is the task's reference, so there is no separate spec to drift from.

``cost`` estimates the fused kernel's FLOPs and HBM bytes (and so its
arithmetic intensity); ``behavioral_hash`` fingerprints what the pipeline
computes (fp32 outputs on a canonical probe), for de-duplication independent
of names, shapes and dtype.

There is no attention, MLA or paged-KV primitive: held-out families cannot be
expressed.

Reference behaviour: kore/openended/grammar.py:82-590.
"""
from __future__ import annotations

import hashlib
import random
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

MAT, ROW = "MAT", "ROW"


@dataclass(frozen=True)
class Primitive:
    name: str
    consumes: str
    produces: str
    aux: Tuple[str, ...] = ()               # "weight" [N_out, N], "bias" [N], "residual" [M, N], "scale" [N]
    flops_per_elem: float = 1.0
    fn: Callable = None                     # fn(x, **aux) on fp32 tensors
    changes_width: bool = False


def _prims() -> Dict[str, Primitive]:
    import torch
    F = torch.nn.functional
    P = [
        Primitive("relu", MAT, MAT, (), 1, lambda x: torch.relu(x)),
        Primitive("gelu", MAT, MAT, (), 8, lambda x: F.gelu(x)),
        Primitive("silu", MAT, MAT, (), 5, lambda x: F.silu(x)),
        Primitive("tanh", MAT, MAT, (), 5, lambda x: torch.tanh(x)),
        Primitive("sigmoid", MAT, MAT, (), 4, lambda x: torch.sigmoid(x)),
        Primitive("square", MAT, MAT, (), 1, lambda x: x * x),
        Primitive("scale2", MAT, MAT, (), 1, lambda x: 2.0 * x),
        Primitive("add_bias", MAT, MAT, ("bias",), 1, lambda x, bias: x + bias),
        Primitive("add_residual", MAT, MAT, ("residual",), 1, lambda x, residual: x + residual),
        Primitive("mul_residual", MAT, MAT, ("residual",), 1, lambda x, residual: x * residual),
        Primitive("rmsnorm", MAT, MAT, ("scale",), 4,
                  lambda x, scale: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * scale),
        Primitive("layernorm", MAT, MAT, (), 7, lambda x: F.layer_norm(x, x.shape[-1:])),
        Primitive("softmax", MAT, MAT, (), 5, lambda x: torch.softmax(x, -1)),
        Primitive("log_softmax", MAT, MAT, (), 5, lambda x: torch.log_softmax(x, -1)),
        Primitive("matmul", MAT, MAT, ("weight",), 0, lambda x, weight: x @ weight.t(), changes_width=True),
        Primitive("row_sum", MAT, ROW, (), 1, lambda x: x.sum(-1)),
        Primitive("row_max", MAT, ROW, (), 1, lambda x: x.amax(-1)),
        Primitive("row_logsumexp", MAT, ROW, (), 4, lambda x: torch.logsumexp(x, -1)),
        Primitive("row_l2", MAT, ROW, (), 2, lambda x: x.pow(2).sum(-1).sqrt()),
    ]
    return {p.name: p for p in P}


_PRIMS: Optional[Dict[str, Primitive]] = None


def primitives() -> Dict[str, Primitive]:
    global _PRIMS
    if _PRIMS is None:
        _PRIMS = _prims()
    return _PRIMS


@dataclass
class Pipeline:
    stages: List[str]
    width_out: int = 0                      # output width of a matmul stage (0 = keep N)

    @property
    def name(self) -> str:
        return "_".join(self.stages)

    def typecheck(self) -> Optional[str]:
        """None when well typed, else the first violation."""
        P = primitives()
        if not self.stages:
            return "empty pipeline"
        cur = MAT
        for i, s in enumerate(self.stages):
            p = P.get(s)
            if p is None:
                return f"unknown primitive {s!r}"
            if cur == ROW:
                return f"{s} follows a terminal row reduction"
            if p.consumes != cur:
                return f"{s} consumes {p.consumes}, got {cur}"
            cur = p.produces
        if sum(1 for s in self.stages if s == "matmul") > 2:
            return "more than two matmuls"
        return None

    @property
    def out_type(self) -> str:
        return primitives()[self.stages[-1]].produces

    def fusion_depth(self) -> int:
        return len(self.stages)

    # ------------------------------------------------------------------ oracle
    def aux_specs(self, M: int, N: int) -> List[Tuple[str, Tuple[int, ...]]]:
        """(name, shape) of every auxiliary input, in argument order."""
        P = primitives()
        out, width = [], N
        for i, s in enumerate(self.stages):
            p = P[s]
            for a in p.aux:
                if a == "weight":
                    w_out = self.width_out or width
                    out.append((f"w{i}", (w_out, width)))
                elif a == "bias" or a == "scale":
                    out.append((f"{a[0]}{i}", (width,)))
                elif a == "residual":
                    out.append((f"r{i}", (M, width)))
            if p.changes_width:
                width = self.width_out or width
        return out

    def build_reference(self) -> Callable:
        """f(x, *aux) in fp32, returned in x's dtype."""
        P = primitives()
        stages = list(self.stages)

        def ref(x, *aux):
            import torch
            y = x.float()
            it = iter(aux)
            for s in stages:
                p = P[s]
                kw = {a: next(it).float() for a in p.aux}
                y = p.fn(y, **kw)
            return y.to(x.dtype) if x.dtype != torch.float32 else y
        return ref

    def build_sampler(self) -> Callable:
        """inputs(dims, seed, device, dtype) -> (x, *aux); GEMM weights are
        scaled by 1/sqrt(K) so deep pipelines stay well conditioned."""
        specs_of = self.aux_specs

        def sample(d: Dict[str, int], seed: int, dev, dt):
            import torch
            g = torch.Generator(device="cpu").manual_seed(int(seed))
            M, N = d["M"], d["N"]
            x = torch.randn(M, N, generator=g)
            out = [x]
            for name, shape in specs_of(M, N):
                t = torch.randn(*shape, generator=g)
                if name.startswith("w"):
                    t = t / shape[1] ** 0.5
                elif name.startswith("s"):
                    t = 1.0 + 0.1 * t
                out.append(t)
            return tuple(t.to(dev).to(dt) for t in out)
        return sample

    # ------------------------------------------------------------------ cost
    def cost(self, M: int, N: int, dtype_bytes: float = 2.0) -> Tuple[float, float]:
        """(FLOPs, HBM bytes) of the fused kernel: inputs and auxiliaries read
        once, the result written once."""
        P = primitives()
        flops, width = 0.0, N
        for s in self.stages:
            p = P[s]
            if s == "matmul":
                w_out = self.width_out or width
                flops += 2.0 * M * width * w_out
                width = w_out
            else:
                flops += p.flops_per_elem * M * width
        elems = M * N + sum(_prod(sh) for _, sh in self.aux_specs(M, N))
        out = M if self.out_type == ROW else M * width
        return flops, (elems + out) * dtype_bytes

    def intensity(self, M: int = 4096, N: int = 4096) -> float:
        f, b = self.cost(M, N)
        return f / b if b else 0.0

    def behavioral_hash(self) -> str:
        """SHA1 of the fp32 outputs on a fixed probe (rounded to 1e-4)."""
        import torch
        x, *aux = self.build_sampler()({"M": 8, "N": 16}, 1234, "cpu", torch.float32)
        y = self.build_reference()(x, *aux)
        q = torch.round(y.double() * 1e4).to(torch.int64)
        return hashlib.sha1(q.numpy().tobytes() + str(tuple(y.shape)).encode()).hexdigest()[:16]


def _prod(shape: Sequence[int]) -> int:
    n = 1
    for v in shape:
        n *= int(v)
    return n


def random_pipeline(rng: random.Random, depth: int, *, allow_matmul: bool = True,
                    terminal: Optional[bool] = None) -> Pipeline:
    """A random well-typed pipeline of ``depth`` stages."""
    P = primitives()
    mat_ops = [n for n, p in P.items() if p.consumes == MAT and p.produces == MAT and
               (allow_matmul or n != "matmul")]
    row_ops = [n for n, p in P.items() if p.produces == ROW]
    end_row = rng.random() < 0.25 if terminal is None else terminal
    stages = [rng.choice(mat_ops) for _ in range(max(1, depth) - (1 if end_row else 0))]
    if end_row:
        stages.append(rng.choice(row_ops))
    return Pipeline(stages)


def lift(operation: str) -> Optional[Pipeline]:
    """A registered operation name as a pipeline, when its words are
    primitives in order (``gemm_bias_gelu`` -> matmul, add_bias, gelu)."""
    P = primitives()
    alias = {"gemm": "matmul", "linear": "matmul", "bias": "add_bias", "residual": "add_residual",
             "rms": "rmsnorm", "ln": "layernorm", "swish": "silu"}
    stages = []
    for w in operation.lower().replace("-", "_").split("_"):
        w = alias.get(w, w)
        if w in P:
            stages.append(w)
    p = Pipeline(stages)
    return p if stages and p.typecheck() is None else None
