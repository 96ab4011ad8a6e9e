"""Four-prong equivalence oracle: a candidate kernel against its reference.

Prongs:

1. random      - ``n_random`` freshly seeded inputs; every element must be
                 within ``atol + rtol |ref|`` and the trial's SNR above
                 ``snr_db_min``;
2. adversarial - the deterministic structured battery (zeros, denormals,
                 huge / tiny magnitudes, activation knots, spikes, ...) per
                 operand slot, plus any folded-in breaking cases;
3. metamorphic - the algebraic relations of the operator class (permutation
                 equivariance, locality, reshape invariance, ...);
4. determinism - ``n_determinism`` runs on identical input must agree.

Comparison is strict on non-finite values: the candidate must put ``nan``
and ``+-inf`` (with the same sign) exactly where the reference does.

The decision is a pure function (:func:`equivalence_verdict`) over
per-prong records, so accept / reject logic is testable without running a
kernel. ``confidence`` = 1 - (1 - p)^m, the probability that a defect
affecting a fraction p of elements (``tol.reference_defect_fraction``) would
have been caught by the m in-tolerance element comparisons of the random
prong. The oracle is tolerance based, not a proof of functional equality.

Reference behaviour: kore/verify/equivalence.py:1-479 (Tolerance, prongs,
pure verdict, (1-p)^m bound).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from . import metamorphic as mm
from .adversarial import battery


@dataclass(frozen=True)
class Tolerance:
    rtol: float = 3e-3
    atol: float = 1e-4
    snr_db_min: float = 50.0
    determinism_rtol: float = 1e-5
    determinism_snr_db_min: float = 80.0
    metamorphic_rtol: float = 6e-3
    metamorphic_snr_db_min: float = 46.0
    reference_defect_fraction: float = 1e-4
    max_violation_fraction: float = 0.0      # fraction of elements allowed outside rtol/atol


_DTYPE_TOL = {
    "fp64": Tolerance(rtol=1e-9, atol=1e-12, snr_db_min=150.0),
    "fp32": Tolerance(),
    "tf32": Tolerance(rtol=2e-2, atol=1e-3, snr_db_min=40.0, metamorphic_rtol=3e-2, metamorphic_snr_db_min=36.0),
    "fp16": Tolerance(rtol=2e-2, atol=1e-3, snr_db_min=38.0, determinism_rtol=1e-3, determinism_snr_db_min=60.0,
                      metamorphic_rtol=3e-2, metamorphic_snr_db_min=34.0, max_violation_fraction=1e-3),
    "bf16": Tolerance(rtol=3e-2, atol=3e-3, snr_db_min=30.0, determinism_rtol=1e-2, determinism_snr_db_min=50.0,
                      metamorphic_rtol=5e-2, metamorphic_snr_db_min=28.0, max_violation_fraction=2e-3),
    "fp8": Tolerance(rtol=1.5e-1, atol=2e-2, snr_db_min=16.0, determinism_rtol=5e-2, determinism_snr_db_min=30.0,
                     metamorphic_rtol=2e-1, metamorphic_snr_db_min=14.0, max_violation_fraction=1e-2),
    "fp4": Tolerance(rtol=3e-1, atol=5e-2, snr_db_min=10.0, determinism_rtol=1e-1, determinism_snr_db_min=20.0,
                     metamorphic_rtol=4e-1, metamorphic_snr_db_min=8.0, max_violation_fraction=2e-2),
}


def tolerance_for(dtype: str) -> Tolerance:
    d = (dtype or "fp32").lower()
    if d.startswith("fp8"):
        d = "fp8"
    if d in ("mxfp4", "nvfp4"):
        d = "fp4"
    return _DTYPE_TOL.get(d, Tolerance())


def snr_db(out: torch.Tensor, ref: torch.Tensor) -> float:
    o, r = out.double(), ref.double()
    fin = torch.isfinite(r)
    if not bool(torch.isfinite(o[fin]).all()):
        return -999.0
    noise = float((o[fin] - r[fin]).norm())
    sig = float(r[fin].norm())
    if noise == 0:
        return 999.0
    return 20 * math.log10(sig / noise) if sig > 0 else -999.0


def false_accept_probability(p_wrong: float, m: int) -> float:
    """Probability that a defect hitting a fraction p of elements survives m
    independent element comparisons."""
    if m <= 0:
        return 1.0
    return math.exp(m * math.log1p(-min(max(p_wrong, 0.0), 1.0 - 1e-16)))


@dataclass
class Comparison:
    """One output compared with its reference."""

    ok: bool
    snr: float
    max_rel: float
    violations: int
    elements: int
    reason: str = ""


def compare(out: torch.Tensor, ref: torch.Tensor, rtol: float, atol: float, snr_min: float,
            max_violation_fraction: float = 0.0) -> Comparison:
    if tuple(out.shape) != tuple(ref.shape):
        return Comparison(False, -999.0, math.inf, ref.numel(), ref.numel(),
                          f"shape {tuple(out.shape)} != {tuple(ref.shape)}")
    o, r = out.detach().double().cpu(), ref.detach().double().cpu()
    n = r.numel()
    nan_r, nan_o = torch.isnan(r), torch.isnan(o)
    inf_r, inf_o = torch.isinf(r), torch.isinf(o)
    if not torch.equal(nan_r, nan_o):
        return Comparison(False, -999.0, math.inf, int((nan_r ^ nan_o).sum()), n, "nan positions differ")
    if not torch.equal(inf_r, inf_o) or not torch.equal(torch.sign(r[inf_r]), torch.sign(o[inf_o])):
        return Comparison(False, -999.0, math.inf, int((inf_r ^ inf_o).sum()) or 1, n, "inf positions or signs differ")
    fin = torch.isfinite(r)
    d = (o[fin] - r[fin]).abs()
    bound = atol + rtol * r[fin].abs()
    viol = int((d > bound).sum())
    rel = float((d / (r[fin].abs() + atol)).max()) if d.numel() else 0.0
    s = snr_db(o, r) if d.numel() else 999.0
    ok = viol <= max_violation_fraction * max(1, int(fin.sum())) and (s >= snr_min or float(d.max() if d.numel()
                                                                                          else 0.0) <= atol)
    reason = "" if ok else (f"{viol} of {n} elements outside rtol={rtol} atol={atol}, SNR {s:.1f} dB")
    return Comparison(ok, s, rel, viol, n, reason)


@dataclass
class ProngResult:
    name: str
    passed: bool
    required: bool = True
    comparisons: int = 0
    worst_snr: float = 999.0
    worst_rel: float = 0.0
    detail: str = ""

    def __bool__(self) -> bool:
        return self.passed


@dataclass
class VerificationResult:
    verified: bool
    confidence: float
    worst_rel: float
    worst_snr: float
    prongs: Dict[str, ProngResult] = field(default_factory=dict)
    first_failure: Optional[str] = None
    false_accept_bound: float = 1.0

    # the earlier verdict record
    @property
    def equivalent(self) -> bool:
        return self.verified

    @property
    def details(self) -> Dict[str, str]:
        return {k: p.detail for k, p in self.prongs.items() if p.detail}

    @property
    def false_accept_at_1pct(self) -> float:
        m = self.prongs["random"].comparisons if "random" in self.prongs else 0
        return false_accept_probability(0.01, m)


Verdict = VerificationResult


def equivalence_verdict(prongs: Sequence[ProngResult], tol: Tolerance) -> VerificationResult:
    """Pure decision over the prong records: verified iff every required
    prong passed; the first failing prong (in order) is reported."""
    by = {p.name: p for p in prongs}
    failing = next((p.name for p in prongs if p.required and not p.passed), None)
    m = by["random"].comparisons if "random" in by else 0
    bound = false_accept_probability(tol.reference_defect_fraction, m)
    worst_snr = min([p.worst_snr for p in prongs] or [999.0])
    worst_rel = max([p.worst_rel for p in prongs] or [0.0])
    return VerificationResult(failing is None, 1.0 - bound, worst_rel, worst_snr, by, failing, bound)


def _as_tuple(x) -> Tuple[torch.Tensor, ...]:
    return tuple(x) if isinstance(x, (tuple, list)) else (x,)


def _outputs(fn: Callable, ins) -> Tuple[torch.Tensor, ...]:
    return _as_tuple(fn(*ins))


def _run_prong(name: str, cases, candidate: Callable, reference: Callable, rtol: float, atol: float,
               snr_min: float, vfrac: float, skip_nonfinite_ref: bool = False) -> ProngResult:
    pr = ProngResult(name, True)
    for label, ins in cases:
        try:
            refs = _outputs(reference, ins)
        except Exception:  # noqa: BLE001 - the reference is undefined here: not a test case
            continue
        if skip_nonfinite_ref and not all(bool(torch.isfinite(r.float()).all()) for r in refs):
            continue
        try:
            outs = _outputs(candidate, ins)
        except Exception as e:  # noqa: BLE001
            pr.passed, pr.detail = False, f"{label}: {type(e).__name__}: {e}"
            break
        if len(outs) != len(refs):
            pr.passed, pr.detail = False, f"{label}: {len(outs)} outputs, expected {len(refs)}"
            break
        for o, r in zip(outs, refs):
            c = compare(o, r, rtol, atol, snr_min, vfrac)
            pr.comparisons += c.elements
            pr.worst_snr = min(pr.worst_snr, c.snr)
            pr.worst_rel = max(pr.worst_rel, c.max_rel)
            if not c.ok:
                pr.passed = False
                pr.detail = f"{label}: {c.reason}"
                break
        if not pr.passed:
            break
    return pr


def verify_equivalence(candidate: Callable, reference: Callable, make_inputs: Callable[[int], Sequence[torch.Tensor]],
                       dtype: str = "fp32", *, family: str = "elementwise", op_class: Optional[str] = None,
                       trials: Optional[int] = None, n_random: int = 16, n_determinism: int = 3,
                       tol: Optional[Tolerance] = None, snr_threshold: Optional[float] = None,
                       adversarial: bool = True, metamorphic: bool = True, determinism: bool = True,
                       adversarial_inputs_fn: Optional[Callable[[Sequence[torch.Tensor]], List]] = None,
                       seed0: int = 0) -> VerificationResult:
    """Run the four prongs. ``make_inputs(seed)`` returns the input tuple;
    ``op_class`` (default: ``family``) picks the metamorphic relations;
    ``adversarial_inputs_fn(inputs)`` adds folded-in breaking cases
    ``[(label, inputs), ...]``."""
    tol = tol or tolerance_for(dtype)
    if snr_threshold is not None:
        tol = replace(tol, snr_db_min=float(snr_threshold))
    n = trials if trials is not None else n_random
    cls = op_class or family
    prongs: List[ProngResult] = []
    rnd = ((f"seed {seed0 + s}", _as_tuple(make_inputs(seed0 + s))) for s in range(n))
    prongs.append(_run_prong("random", rnd, candidate, reference, tol.rtol, tol.atol, tol.snr_db_min,
                             tol.max_violation_fraction))
    if adversarial:
        base = _as_tuple(make_inputs(seed0 + 1000))
        cases = list(battery(base, dtype=dtype))
        if adversarial_inputs_fn is not None:
            cases += list(adversarial_inputs_fn(base))
        prongs.append(_run_prong("adversarial", cases, candidate, reference, tol.rtol, tol.atol,
                                 tol.snr_db_min, tol.max_violation_fraction, skip_nonfinite_ref=False))
    if metamorphic:
        ins = _as_tuple(make_inputs(seed0 + 2000))
        pr = ProngResult("metamorphic", True)
        for rel in mm.relations_for(cls):
            try:
                good, why = rel(candidate, *ins, rtol=tol.metamorphic_rtol)
            except Exception as e:  # noqa: BLE001
                good, why = False, f"{type(e).__name__}: {e}"
            pr.comparisons += 1
            if not good:
                pr.passed, pr.detail = False, why
                break
        prongs.append(pr)
    if determinism:
        ins = _as_tuple(make_inputs(seed0 + 3000))
        pr = ProngResult("determinism", True)
        try:
            first = _outputs(candidate, ins)
            for _ in range(max(1, n_determinism - 1)):
                again = _outputs(candidate, ins)
                for a, b in zip(first, again):
                    if torch.equal(a, b):
                        continue
                    c = compare(b, a, tol.determinism_rtol, 0.0, tol.determinism_snr_db_min)
                    if not c.ok:
                        pr.passed, pr.detail = False, "outputs differ between identical runs: " + c.reason
                        break
                if not pr.passed:
                    break
        except Exception as e:  # noqa: BLE001
            pr.passed, pr.detail = False, f"{type(e).__name__}: {e}"
        prongs.append(pr)
    return equivalence_verdict(prongs, tol)
