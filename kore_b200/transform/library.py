"""The rewrite library (Triton-source transforms for B200 candidates).

Exact: double / halve BM, BN, BK, BLOCK; num_warps 4<->8; num_stages
2->3->4; add ``tl.multiple_of`` hints; switch ``tl.exp`` to ``tl.exp2`` with
a log2(e) pre-scale (exact up to rounding). Approximate: fp16 products with
fp32 accumulation (eps 1e-3), drop the max-subtraction of a softmax on
bounded inputs (eps 1e-2). Reference parity: kore/transform/library.py:737-744
(>= 12 rewrites) and discover.py:311 (knob sweeps)."""
from __future__ import annotations

import re
from typing import List, Optional

from .calculus import Transformation, replace_int_kwarg


def _pow2_ok(n: int) -> bool:
    return n >= 16 and n <= 1024 and (n & (n - 1)) == 0


def _scale(name, f):
    return replace_int_kwarg(name, lambda v: f(v) if _pow2_ok(f(v)) else v)


def _exp2(src: str) -> Optional[str]:
    if "tl.exp(" not in src:
        return None
    return src.replace("tl.exp(", "tl.exp2(1.4426950408889634 * ")


def _hint(src: str) -> Optional[str]:
    m = re.search(r"(\n(\s+)cols = tl\.arange\(0, BLOCK\)\n)", src)
    if not m or "multiple_of" in src:
        return None
    ind = m.group(2)
    return src.replace(m.group(1), m.group(1) + f"{ind}cols = tl.max_contiguous(tl.multiple_of(cols, 16), 16)\n", 1)


def _stages(src: str) -> Optional[str]:
    m = re.search(r"\bnum_stages\s*=\s*(\d+)", src)
    if m:
        v = int(m.group(1))
        return None if v >= 4 else src[: m.start(1)] + str(v + 1) + src[m.end(1):]
    m = re.search(r"(\w+\[\([^\]]*\)\]\([^)]*)(\))", src)
    return None if not m else src[: m.end(1)] + ", num_stages=3" + src[m.end(1):]


def _warps(target):
    def rw(src: str) -> Optional[str]:
        m = re.search(r"\bnum_warps\s*=\s*(\d+)", src)
        if m:
            return None if int(m.group(1)) == target else src[: m.start(1)] + str(target) + src[m.end(1):]
        m = re.search(r"(\w+\[\([^\]]*\)\]\([^)]*)(\))", src)
        return None if not m else src[: m.end(1)] + f", num_warps={target}" + src[m.end(1):]
    return rw


def _fp16_products(src: str) -> Optional[str]:
    if "tl.dot(a, b)" not in src:
        return None
    return src.replace("tl.dot(a, b)", "tl.dot(a.to(tl.float16), b.to(tl.float16), out_dtype=tl.float32)")


LIBRARY: List[Transformation] = [
    Transformation("bm_x2", "exact", _scale("BM", lambda v: v * 2)),
    Transformation("bm_half", "exact", _scale("BM", lambda v: v // 2)),
    Transformation("bn_x2", "exact", _scale("BN", lambda v: v * 2)),
    Transformation("bn_half", "exact", _scale("BN", lambda v: v // 2)),
    Transformation("bk_x2", "exact", _scale("BK", lambda v: v * 2)),
    Transformation("bk_half", "exact", _scale("BK", lambda v: v // 2)),
    Transformation("block_x2", "exact", _scale("BLOCK", lambda v: v * 2)),
    Transformation("block_half", "exact", _scale("BLOCK", lambda v: v // 2)),
    Transformation("warps_4", "exact", _warps(4)),
    Transformation("warps_8", "exact", _warps(8)),
    Transformation("stages_up", "exact", _stages),
    Transformation("contiguity_hint", "exact", _hint),
    Transformation("exp_to_exp2", "exact", _exp2),
    Transformation("fp16_products", "approx", _fp16_products, eps=1e-3),
]
_BY_NAME = {t.name: t for t in LIBRARY}


def get_transform(name: str) -> Optional[Transformation]:
    return _BY_NAME.get(name)


def admissible(src: str) -> List[Transformation]:
    return [t for t in LIBRARY if t.apply(src) is not None]


def discover_knobs(src: str) -> List[Transformation]:
    """Knob sweeps discovered from integer constexpr kwargs in the source."""
    out = []
    for name in sorted(set(re.findall(r"\b([A-Z][A-Z_]{1,15})\s*=\s*\d+", src))):
        if name in ("BM", "BN", "BK", "BLOCK"):
            continue
        out.append(Transformation(f"{name.lower()}_x2", "exact", _scale(name, lambda v: v * 2)))
        out.append(Transformation(f"{name.lower()}_half", "exact", _scale(name, lambda v: v // 2)))
    return out
