"""The rewrite library: typed Triton-source rewrites for B200 candidates.

Exact (bit-preserving) families:
  set_num_stages      software-pipelining depth of the launch (2..5)
  set_num_ctas        thread-block cluster size of the launch (1, 2)
  swizzle_group_m     L2 super-grouping of program ids (existing GROUP_M knob)
  vectorize_loads     tl.multiple_of / tl.max_contiguous hints on the column range
  add_mask_boundary   guard an unmasked load / store with the mask already in scope
  reorder_loads       swap two adjacent data-independent tl.load statements
  warp_specialize     producer/consumer warp specialisation of the K loop (tl.range)
Approximate families (spend epsilon):
  set_num_warps       may reassociate cross-warp reductions            eps 0.005
  fp32_accumulator    low-precision tl.zeros accumulator -> fp32       eps 1e-6
  retile_block        halve / double a BLOCK_* constexpr               eps 0.02 (K-like: 0.06)
  split_k             split the K loop over a grid axis, atomic adds   eps 0.05 x ways / 2
  downcast_dtype      cast tl.dot operands to bf16 / fp16 / fp8        eps 0.03 / 0.05 / 0.15
  reassociate_reduction  acc += tl.dot(a, b)  ->  acc = tl.dot(a, b, acc)   eps 0.01
  fast_math_recip     1.0 / x -> non-IEEE division                      eps 0.03
  exp_to_exp2         tl.exp(x) -> tl.exp2(x * log2 e)                   eps 1e-6
  rsqrt               1.0 / tl.sqrt(x) -> tl.rsqrt(x)                    eps 0.01

``LIBRARY`` holds the families; :func:`actions_for` / :func:`admissible`
enumerate concrete actions. Every rewrite is a pure function of the source
text (regular expressions over the canonical Triton idioms the task seeds and
the policy's kernels use); a rewrite that does not recognise its idiom
returns None instead of guessing.

Reference behaviour: kore/transform/library.py:1-744 (13 typed rewrites keyed
off the launch-knob conventions), retargeted to Triton on sm_100a (clusters,
warp specialisation, fp8 operands instead of the reference's gfx950 knobs).
"""
from __future__ import annotations

import re
from typing import Dict, List, Optional

from .budget import APPROX, EXACT
from .calculus import Action, Params, Transformation, find_int_kwarg, set_int_kwarg

# ----------------------------------------------------------------------------- helpers
_LAUNCH = re.compile(r"(\w+\[[^\]]*\]\()")       # kernel[grid](


def _launch_spans(src: str) -> List[tuple]:
    """(start, end) of each ``kernel[grid](...)`` call, end = index of its ')'."""
    out = []
    for m in _LAUNCH.finditer(src):
        depth, i = 1, m.end()
        while i < len(src) and depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        if depth == 0:
            out.append((m.start(), i - 1))
    return out


def _set_launch_kwarg(src: str, name: str, value) -> Optional[str]:
    """Set ``name=value`` on every kernel launch (add it where missing)."""
    spans = _launch_spans(src)
    if not spans:
        return None
    out, last = [], 0
    for a, b in spans:
        call = src[a:b]
        if re.search(rf"\b{name}\s*=", call):
            call = re.sub(rf"\b({name}\s*=\s*)[^,)\n]+", rf"\g<1>{value}", call, count=1)
        else:
            call = call.rstrip() + f", {name}={value}"
        out.append(src[last:a] + call)
        last = b
    out.append(src[last:])
    return "".join(out)


def _launch_kwarg(src: str, name: str) -> Optional[int]:
    for a, b in _launch_spans(src):
        m = re.search(rf"\b{name}\s*=\s*(\d+)", src[a:b])
        if m:
            return int(m.group(1))
    return None


def _is_triton(src: str) -> bool:
    return "@triton.jit" in src


# ----------------------------------------------------------------------------- exact families
def _stages_domain(src: str) -> List[Params]:
    cur = _launch_kwarg(src, "num_stages")
    return [{"n": n} for n in (2, 3, 4, 5) if n != cur]


def _stages(src: str, n: int = 3) -> Optional[str]:
    if not _is_triton(src) or "for " not in src:
        return None
    return _set_launch_kwarg(src, "num_stages", n)


def _ctas_domain(src: str) -> List[Params]:
    cur = _launch_kwarg(src, "num_ctas") or 1
    return [{"n": n} for n in (1, 2) if n != cur]


def _ctas(src: str, n: int = 2) -> Optional[str]:
    if not _is_triton(src) or "tl.dot(" not in src:
        return None
    return _set_launch_kwarg(src, "num_ctas", n)


def _group_domain(src: str) -> List[Params]:
    cur = find_int_kwarg(src, "GROUP_M")
    return [] if cur is None else [{"g": g} for g in (4, 8, 16) if g != cur]


def _group(src: str, g: int = 8) -> Optional[str]:
    return set_int_kwarg(src, "GROUP_M", g) if find_int_kwarg(src, "GROUP_M") is not None else None


def _vectorize(src: str, width: int = 16) -> Optional[str]:
    m = re.search(r"\n([ \t]+)(\w+) = tl\.arange\(0, (\w+)\)\n", src)
    if not m or "multiple_of" in src:
        return None
    ind, var = m.group(1), m.group(2)
    hint = f"{ind}{var} = tl.max_contiguous(tl.multiple_of({var}, {width}), {width})\n"
    return src[: m.end()] + hint + src[m.end():]


def _vec_domain(src: str) -> List[Params]:
    return [{"width": w} for w in (8, 16)]


_UNMASKED = re.compile(r"tl\.(load|store)\(([^()\n]*(?:\([^()\n]*\)[^()\n]*)*)\)")


def _mask_boundary(src: str) -> Optional[str]:
    """Add ``mask=<m>`` to the first unmasked load/store whose pointer uses the
    same offset variable as an existing ``<m> = <var> < ...`` guard."""
    guards = dict((v, g) for g, v in re.findall(r"\n\s*(\w+)\s*=\s*(\w+)\s*<\s*\w+", src))
    if not guards:
        return None
    for m in _UNMASKED.finditer(src):
        args = m.group(2)
        if "mask=" in args:
            continue
        for var, g in guards.items():
            if re.search(rf"\b{var}\b", args.split(",")[0]):
                extra = f", mask={g}" + (", other=0.0" if m.group(1) == "load" else "")
                return src[: m.end(2)] + extra + src[m.end(2):]
    return None


def _reorder_loads(src: str) -> Optional[str]:
    lines = src.split("\n")
    for i in range(len(lines) - 1):
        a, b = lines[i], lines[i + 1]
        ma = re.match(r"^([ \t]+)(\w+)\s*=\s*tl\.load\(", a)
        mb = re.match(r"^([ \t]+)(\w+)\s*=\s*tl\.load\(", b)
        if ma and mb and ma.group(1) == mb.group(1):
            if re.search(rf"\b{ma.group(2)}\b", b.split("=", 1)[1]):
                continue                        # b reads what a loads: not independent
            lines[i], lines[i + 1] = b, a
            return "\n".join(lines)
    return None


def _warp_specialize(src: str) -> Optional[str]:
    if "tl.dot(" not in src or "warp_specialize" in src:
        return None
    m = re.search(r"for (\w+) in range\(([^\n]*)\):", src)
    if not m:
        return None
    return src[: m.start()] + f"for {m.group(1)} in tl.range({m.group(2)}, warp_specialize=True):" + src[m.end():]


# ----------------------------------------------------------------------------- approximate families
def _warps_domain(src: str) -> List[Params]:
    cur = _launch_kwarg(src, "num_warps") or 4
    return [{"n": n} for n in (4, 8, 2, 16) if n != cur]


def _warps(src: str, n: int = 8) -> Optional[str]:
    return _set_launch_kwarg(src, "num_warps", n) if _is_triton(src) else None


def _warps_eps(p: Params) -> float:
    return 0.005          # a cross-warp reduction may be summed in another order


def _fp32_acc(src: str) -> Optional[str]:
    pat = re.compile(r"(tl\.zeros\([^\n]*dtype\s*=\s*)tl\.(float16|bfloat16)")
    return pat.sub(r"\1tl.float32", src, count=1) if pat.search(src) else None


_KLIKE = ("BK", "BLOCK_K", "BLOCK_SIZE_K")


def _retile_domain(src: str) -> List[Params]:
    out = []
    for name in sorted(set(re.findall(r"\b(B[MNK]|BLOCK(?:_SIZE)?(?:_[MNK])?)\s*=\s*\d+", src))):
        for f in ("x2", "half"):
            out.append({"name": name, "f": f})
    return out


def _retile(src: str, name: str = "BLOCK", f: str = "x2") -> Optional[str]:
    v = find_int_kwarg(src, name)
    if v is None:
        return None
    new = v * 2 if f == "x2" else v // 2
    if new < 16 or new > 1024 or new & (new - 1):
        return None
    return set_int_kwarg(src, name, new)


def _retile_eps(p: Params) -> float:
    return 0.06 if p.get("name") in _KLIKE else 0.02


def _split_top(s: str) -> List[str]:
    """Split on the commas that are not inside parentheses."""
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
            continue
        depth += {"(": 1, ")": -1, "[": 1, "]": -1}.get(ch, 0)
        cur += ch
    out.append(cur.strip())
    return out


_KLOOP = re.compile(r"for (\w+) in range\(0, (\w+), (\w+)\):")


def _split_k(src: str, ways: int = 2) -> Optional[str]:
    """Canonical GEMM: K loop ``for k in range(0, K, BK)`` with one ``tl.store``
    of the accumulator; each of ``ways`` programs on grid axis 2 sums a strided
    share of the K blocks and atomically adds its partial tile. The output must
    start at zero, so ``torch.empty`` allocations become ``torch.zeros``."""
    if "SPLIT_K" in src or "tl.dot(" not in src:
        return None
    m = _KLOOP.search(src)
    st = re.search(r"tl\.store\(([^\n]*)acc(\.to\([^)]*\))?([^\n]*)\)\n", src)
    grid = re.search(r"(\w+)\[\(([^\]]*?)\)\]\(", src)
    if not m or not st or not grid:
        return None
    kv, K, BK = m.groups()
    parts = [p for p in _split_top(grid.group(2)) if p]
    if len(parts) != 2:
        return None
    out = src[: m.start()] + (f"for {kv} in range(tl.program_id(2) * {BK}, {K}, {BK} * SPLIT_K):") + src[m.end():]
    st = re.search(r"tl\.store\(([^\n]*)acc(\.to\([^)]*\))?([^\n]*)\)\n", out)
    out = out[: st.start()] + "tl.atomic_add(" + st.group(1) + "acc" + (st.group(3) or "") + ")\n" + out[st.end():]
    out = re.sub(r"(BK: tl\.constexpr)", r"\1, SPLIT_K: tl.constexpr", out, count=1)
    grid = re.search(r"(\w+)\[\(([^\]]*?)\)\]\(", out)
    out = out[: grid.start(2)] + f"{parts[0]}, {parts[1]}, {ways}" + out[grid.end(2):]
    call = _launch_spans(out)
    if not call:
        return None
    a, b = call[0]
    out = out[:b] + f", SPLIT_K={ways}" + out[b:]
    out = out.replace("torch.empty_like(", "torch.zeros_like(").replace("torch.empty(", "torch.zeros(")
    return out


def _split_conditions(src: str, p: Params) -> List[str]:
    why = []
    if p.get("ways", 2) not in (2, 4, 8):
        why.append("ways must be 2, 4 or 8")
    if "bias" in src.lower() or "residual" in src.lower():
        why.append("an epilogue term would be added once per split")
    return why


_DOWN = {"bf16": ("tl.bfloat16", 0.03), "fp16": ("tl.float16", 0.05), "fp8": ("tl.float8e4nv", 0.15)}


def _downcast(src: str, to: str = "bf16") -> Optional[str]:
    m = re.search(r"tl\.dot\((\w+), (\w+)", src)
    if not m or ".to(" in src[m.start(): m.start() + 60]:
        return None
    ty = _DOWN[to][0]
    return src[: m.start()] + f"tl.dot({m.group(1)}.to({ty}), {m.group(2)}.to({ty})" + src[m.end():]


def _reassoc(src: str) -> Optional[str]:
    pat = re.compile(r"(\w+) \+= tl\.dot\(([^()\n]*(?:\([^()\n]*\)[^()\n]*)*)\)")
    m = pat.search(src)
    if not m:
        return None
    return src[: m.start()] + f"{m.group(1)} = tl.dot({m.group(2)}, {m.group(1)})" + src[m.end():]


def _fast_recip(src: str) -> Optional[str]:
    pat = re.compile(r"\b1\.0\s*/\s*(\(?[\w.]+(?:\([^()\n]*\))?\)?)")
    m = pat.search(src)
    if not m or "tl.sqrt" in m.group(1) or not _is_triton(src):
        return None
    return src[: m.start()] + f"tl.fdiv(1.0, {m.group(1)}, ieee_rounding=False)" + src[m.end():]


def _exp2(src: str) -> Optional[str]:
    if "tl.exp(" not in src:
        return None
    return src.replace("tl.exp(", "tl.exp2(1.4426950408889634 * ")


def _rsqrt(src: str) -> Optional[str]:
    pat = re.compile(r"1\.0\s*/\s*tl\.sqrt\(")
    if not pat.search(src):
        return None
    return pat.sub("tl.rsqrt(", src, count=1)


# ----------------------------------------------------------------------------- CUDA C++ sources
_KERNEL_SIG = re.compile(r"__global__\s+(?:__launch_bounds__\([^)]*\)\s+)?void\s+(\w+)\s*\(([^)]*)\)")


def _is_cuda(src: str) -> bool:
    return "__global__" in src


def _launch_bounds_domain(src: str) -> List[Params]:
    if not _is_cuda(src):
        return []
    m = re.search(r"<<<[^,>]+,\s*(\d+)", src) or re.search(r"blockDim\s*=\s*dim3\((\d+)", src)
    n = int(m.group(1)) if m else 256
    return [{"threads": n, "min_blocks": b} for b in (1, 2)]


def _launch_bounds(src: str, threads: int = 256, min_blocks: int = 1) -> Optional[str]:
    """Add (or replace) ``__launch_bounds__(threads, min_blocks)`` on the first
    kernel: register allocation only, the arithmetic is unchanged. The launch
    must not use more than ``threads`` threads per block (side condition)."""
    m = re.search(r"__global__\s+(__launch_bounds__\([^)]*\)\s+)?void", src)
    if not m:
        return None
    lb = f"__launch_bounds__({int(threads)}, {int(min_blocks)}) "
    if m.group(1):
        return src[: m.start(1)] + lb + src[m.end(1):]
    return src[: m.start()] + "__global__ " + lb + "void" + src[m.end():]


def _launch_bounds_conditions(src: str, p: Params) -> List[str]:
    out = []
    for n in re.findall(r"<<<[^,>]+,\s*(\d+)", src):
        if int(n) > int(p.get("threads", 256)):
            out.append("launch uses more threads than the bound")
    return out


def _restrict(src: str) -> Optional[str]:
    """Mark the first kernel's pointer parameters ``__restrict__`` (lets the
    compiler use the read-only path and reorder loads)."""
    m = _KERNEL_SIG.search(src)
    if not m or "__restrict__" in m.group(2):
        return None
    params = m.group(2).split(",")
    new, changed = [], False
    for prm in params:
        if "*" in prm and "__restrict__" not in prm:
            head, _, name = prm.rpartition("*")
            new.append(f"{head}* __restrict__{name if name.startswith(' ') else ' ' + name.strip()}")
            changed = True
        else:
            new.append(prm)
    if not changed:
        return None
    return src[: m.start(2)] + ",".join(new) + src[m.end(2):]


def _restrict_conditions(src: str, p: Params) -> List[str]:
    """Legal only when no two pointer arguments of a launch are the same buffer."""
    for args in re.findall(r"<<<[^>]*>>>\s*\(([^;]*)\)", src):
        names = [a.strip() for a in args.split(",") if a.strip()]
        if len(names) != len(set(names)):
            return ["a launch passes the same argument twice (possible aliasing)"]
    return []


def _unroll(src: str) -> Optional[str]:
    """``#pragma unroll`` on the first constant-trip ``for`` loop without one."""
    for m in re.finditer(r"(?m)^([ \t]*)for\s*\(\s*int\s+\w+\s*=\s*0\s*;\s*\w+\s*<\s*(\d+|[A-Z_][A-Z0-9_]*)\s*;", src):
        prev = src[: m.start()].rstrip().splitlines()[-1:] if src[: m.start()].strip() else []
        if prev and prev[0].strip().startswith("#pragma unroll"):
            continue
        return src[: m.start()] + f"{m.group(1)}#pragma unroll\n" + src[m.start():]
    return None


def _one(params: Params):
    return lambda src: [dict(params)]


LIBRARY: List[Transformation] = [
    Transformation("set_num_stages", EXACT, _stages, knob="num_stages", domain=_stages_domain,
                   doc="software-pipelining depth of the K loop"),
    Transformation("set_num_ctas", EXACT, _ctas, knob="num_ctas", domain=_ctas_domain,
                   doc="thread-block cluster size"),
    Transformation("swizzle_group_m", EXACT, _group, knob="GROUP_M", domain=_group_domain,
                   doc="L2 super-grouping of output tiles"),
    Transformation("vectorize_loads", EXACT, _vectorize, knob="vectorize", domain=_vec_domain,
                   doc="contiguity / divisibility hints (compiler only)"),
    Transformation("add_mask_boundary", EXACT, _mask_boundary, knob="mask",
                   doc="reuse an in-scope guard on an unmasked access"),
    Transformation("reorder_loads", EXACT, _reorder_loads, knob="layout",
                   doc="swap two adjacent independent loads"),
    Transformation("warp_specialize", EXACT, _warp_specialize, knob="warp_specialize",
                   doc="producer / consumer warps for the K loop"),
    Transformation("set_num_warps", APPROX, _warps, knob="num_warps", domain=_warps_domain, eps_fn=_warps_eps,
                   side_conditions=lambda s, p: [] if p.get("n", 8) in (1, 2, 4, 8, 16) else ["warps"],
                   doc="warp count; may reassociate a cross-warp reduction"),
    Transformation("fp32_accumulator", APPROX, _fp32_acc, eps=1e-6, knob="accumulator",
                   doc="fp32 accumulator (more precise, not bit-identical)"),
    Transformation("retile_block", APPROX, _retile, knob="block", domain=_retile_domain, eps_fn=_retile_eps,
                   doc="re-tile a BLOCK_* constexpr"),
    Transformation("split_k", APPROX, _split_k, knob="split_k", domain=lambda s: [{"ways": w} for w in (2, 4)],
                   eps_fn=lambda p: 0.05 * p.get("ways", 2) / 2, side_conditions=_split_conditions,
                   doc="split the K reduction over grid axis 2 with atomic partials"),
    Transformation("downcast_dtype", APPROX, _downcast, knob="dtype",
                   domain=lambda s: [{"to": t} for t in ("bf16", "fp16", "fp8")],
                   eps_fn=lambda p: _DOWN[p.get("to", "bf16")][1], doc="cast the dot operands, fp32 accumulate"),
    Transformation("reassociate_reduction", APPROX, _reassoc, eps=0.01, knob="reduction",
                   doc="accumulate inside tl.dot"),
    Transformation("fast_math_recip", APPROX, _fast_recip, eps=0.03, knob="fast_math",
                   doc="non-IEEE reciprocal"),
    Transformation("exp_to_exp2", APPROX, _exp2, eps=1e-6, knob="fast_math",
                   doc="exp through exp2 with a log2(e) pre-scale (rounding differs)"),
    Transformation("rsqrt", APPROX, _rsqrt, eps=0.01, knob="fast_math", doc="1/sqrt -> rsqrt"),
    Transformation("cuda_launch_bounds", EXACT, _launch_bounds, knob="launch_bounds", domain=_launch_bounds_domain,
                   side_conditions=_launch_bounds_conditions,
                   doc="__launch_bounds__(threads, min blocks): register budget of a CUDA kernel"),
    Transformation("cuda_restrict", EXACT, _restrict, knob="aliasing", side_conditions=_restrict_conditions,
                   doc="__restrict__ pointer parameters (no two arguments alias)"),
    Transformation("cuda_unroll", EXACT, _unroll, knob="unroll",
                   doc="#pragma unroll on a constant-trip loop"),
]
EXACT_LIBRARY = [t for t in LIBRARY if t.kind == EXACT]
APPROX_LIBRARY = [t for t in LIBRARY if t.kind == APPROX]
_BY_NAME: Dict[str, Transformation] = {t.name: t for t in LIBRARY}


def get_transform(name: str):
    """A family by name, or one concrete action written ``family(k=v,...)``."""
    if name in _BY_NAME:
        return _BY_NAME[name]
    m = re.match(r"^(\w+)\((.*)\)$", name or "")
    if not m or m.group(1) not in _BY_NAME:
        return None
    params: Params = {}
    for kv in filter(None, m.group(2).split(",")):
        k, v = kv.split("=", 1)
        params[k.strip()] = int(v) if v.strip().lstrip("-").isdigit() else v.strip()
    return Action(_BY_NAME[m.group(1)], params)


def actions_for(src: str, library: Optional[List[Transformation]] = None) -> List[Action]:
    return [a for t in (library or LIBRARY) for a in t.actions(src)]


def admissible(src: str, budget=None) -> List[Action]:
    """Concrete actions that apply to ``src`` (within ``budget`` when given)."""
    from .calculus import admissible_actions
    return admissible_actions(src, LIBRARY, budget)
