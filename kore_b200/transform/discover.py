"""Self-extending rewrite library (opt-in; the curated ``LIBRARY`` is never
mutated).

``discover_transforms(src)`` reads a kernel and proposes candidate rewrite
families the curated library does not cover:

* knob sweeps over every integer ``tl.constexpr`` launch argument that is not
  already a curated knob (halve / double within powers of two);
* vector widths for the contiguity hint (4, 8, 16, 32);
* fusion of an elementwise epilogue: a ``y = f(x)`` line right before a store
  of ``y`` is folded into the store (fewer live registers).

Every proposal is typed ``approx`` with a conservative epsilon, because
nothing in this module proves it bit-preserving; the environment's SNR gate
decides. ``merge_transforms`` de-duplicates by name (curated first);
``extend_library`` returns a new list and refuses proposals whose name
collides with a curated family.

Reference behaviour: kore/transform/discover.py:1-426.
"""
from __future__ import annotations

import re
from typing import Iterable, List, Optional, Sequence

from .budget import APPROX
from .calculus import Params, Transformation, find_int_kwarg, set_int_kwarg
from .library import LIBRARY

DISCOVERED_EPS = 0.02
_CURATED_KNOBS = {"BM", "BN", "BK", "BLOCK", "BLOCK_M", "BLOCK_N", "BLOCK_K", "GROUP_M", "SPLIT_K"}


def _pow2(n: int) -> bool:
    return 1 <= n <= 4096 and (n & (n - 1)) == 0


def _knob_family(name: str) -> Transformation:
    def rw(src: str, f: str = "x2") -> Optional[str]:
        v = find_int_kwarg(src, name)
        if v is None:
            return None
        new = v * 2 if f == "x2" else v // 2
        return set_int_kwarg(src, name, new) if _pow2(new) and new != v else None

    return Transformation(f"sweep_{name.lower()}", APPROX, rw, eps=DISCOVERED_EPS, knob=name,
                          domain=lambda s: [{"f": "x2"}, {"f": "half"}],
                          doc=f"discovered: halve / double the {name} launch constant")


def _vector_family() -> Transformation:
    def rw(src: str, width: int = 16) -> Optional[str]:
        m = re.search(r"tl\.max_contiguous\(tl\.multiple_of\((\w+), (\d+)\), (\d+)\)", src)
        if not m or int(m.group(2)) == width:
            return None
        return src[: m.start()] + f"tl.max_contiguous(tl.multiple_of({m.group(1)}, {width}), {width})" + src[m.end():]

    return Transformation("discovered_vector_width", APPROX, rw, eps=DISCOVERED_EPS, knob="vectorize",
                          domain=lambda s: [{"width": w} for w in (4, 8, 16, 32)],
                          doc="discovered: other contiguity widths")


_EPI = re.compile(r"\n([ \t]+)(\w+) = ([^\n]+)\n\1tl\.store\(([^,\n]+), \2([,)])")


def _fuse_family() -> Transformation:
    def rw(src: str) -> Optional[str]:
        m = _EPI.search(src)
        if not m:
            return None
        ind, var, expr, ptr, tail = m.groups()
        a = src.rfind("\ndef ", 0, m.start())
        b = src.find("\ndef ", m.end())
        body = src[a: b if b >= 0 else len(src)]
        if len(re.findall(rf"\b{var}\b", body)) != 2:     # defined once, used only by the store
            return None
        return src[: m.start()] + f"\n{ind}tl.store({ptr}, ({expr}){tail}" + src[m.end():]

    return Transformation("fuse_epilogue", APPROX, rw, eps=DISCOVERED_EPS, knob="fusion",
                          doc="discovered: fold a one-use elementwise epilogue into its store")


def discover_transforms(src: str) -> List[Transformation]:
    out: List[Transformation] = []
    consts = re.findall(r"\b([A-Z][A-Z0-9_]{1,20})\s*:\s*tl\.constexpr", src)
    for name in sorted(set(consts)):
        if name in _CURATED_KNOBS or find_int_kwarg(src, name) is None:
            continue
        fam = _knob_family(name)
        if any(a.apply(src) is not None for a in fam.actions(src)):
            out.append(fam)
    vec = _vector_family()
    if any(a.apply(src) is not None for a in vec.actions(src)):
        out.append(vec)
    fuse = _fuse_family()
    if fuse.apply(src) is not None:
        out.append(fuse)
    return out


def merge_transforms(*groups: Iterable[Transformation]) -> List[Transformation]:
    seen, out = set(), []
    for g in groups:
        for t in g:
            if t.name not in seen:
                seen.add(t.name)
                out.append(t)
    return out


def extend_library(src: str, library: Sequence[Transformation] = LIBRARY, *, enabled: bool = False
                   ) -> List[Transformation]:
    """``library`` plus this source's discovered families (only when enabled)."""
    base = list(library)
    if not enabled:
        return base
    curated = {t.name for t in base}
    return merge_transforms(base, [t for t in discover_transforms(src) if t.name not in curated])


def describe(t: Transformation, src: str) -> List[Params]:
    return [a.params for a in t.actions(src) if a.apply(src) is not None]
