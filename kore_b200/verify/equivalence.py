"""Multi-prong equivalence verdict of a candidate against an oracle.

Prongs: (1) m random trials (fresh seeds), (2) the adversarial battery,
(3) metamorphic relations matching the operator family, (4) determinism
(identical inputs give identical outputs across runs). The verdict carries
the worst SNR, per-prong results and the probability that an implementation
which is wrong on a fraction p of inputs passes all m random trials,
(1 - p)^m. Reference parity: kore/verify/equivalence.py:357-479.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, Optional, Sequence

import torch

from . import metamorphic as mm
from .adversarial import battery


def snr_db(out: torch.Tensor, ref: torch.Tensor) -> float:
    o, r = out.float(), ref.float()
    if not torch.isfinite(o).all() and torch.isfinite(r).all():
        return -999.0
    noise = (o - r).norm().item()
    sig = r.norm().item()
    if noise == 0:
        return 999.0
    return 20 * math.log10(sig / noise) if sig > 0 else -999.0


def false_accept_probability(p_wrong: float, m: int) -> float:
    return (1.0 - p_wrong) ** m


@dataclass
class Verdict:
    equivalent: bool
    worst_snr: float
    prongs: Dict[str, bool] = field(default_factory=dict)
    details: Dict[str, str] = field(default_factory=dict)
    trials: int = 0
    false_accept_at_1pct: float = 1.0


def verify_equivalence(candidate: Callable, oracle: Callable, make_inputs: Callable[[int], Sequence[torch.Tensor]],
                       *, family: str = "elementwise", trials: int = 5, snr_threshold: float = 30.0,
                       adversarial: bool = True, metamorphic: bool = True, determinism: bool = True) -> Verdict:
    worst = 999.0
    prongs: Dict[str, bool] = {}
    details: Dict[str, str] = {}
    ok = True
    for s in range(trials):
        ins = make_inputs(s)
        try:
            v = snr_db(candidate(*ins), oracle(*ins))
        except Exception as e:  # noqa: BLE001
            v = -999.0
            details["random"] = f"{type(e).__name__}: {e}"
        worst = min(worst, v)
    prongs["random"] = worst >= snr_threshold
    if adversarial:
        adv_ok = True
        for name, ins in battery(make_inputs(1000)):
            try:
                ref = oracle(*ins)
                if not torch.isfinite(ref.float()).all():
                    continue
                v = snr_db(candidate(*ins), ref)
            except Exception as e:  # noqa: BLE001
                v = -999.0
                details[f"adv_{name}"] = str(e)
            if v < snr_threshold and ref.float().abs().max() > 0:
                adv_ok = False
                details.setdefault("adversarial", name)
        prongs["adversarial"] = adv_ok
    if metamorphic:
        ins = make_inputs(2000)
        checks = []
        if family in ("elementwise", "unary", "binary"):
            checks = [mm.elementwise_permutation, mm.elementwise_locality]
        elif family in ("reduce", "norm"):
            checks = [mm.reduction_row_permutation]
        res = True
        for c in checks:
            try:
                good, why = c(candidate, *ins)
            except Exception as e:  # noqa: BLE001
                good, why = False, str(e)
            if not good:
                res = False
                details["metamorphic"] = why
        prongs["metamorphic"] = res
    if determinism:
        ins = make_inputs(3000)
        try:
            a, b = candidate(*ins), candidate(*ins)
            prongs["determinism"] = snr_db(a, b) >= snr_threshold + 10 or torch.equal(a, b)
        except Exception as e:  # noqa: BLE001
            prongs["determinism"] = False
            details["determinism"] = str(e)
    ok = all(prongs.values())
    return Verdict(ok, worst, prongs, details, trials, false_accept_probability(0.01, trials))
