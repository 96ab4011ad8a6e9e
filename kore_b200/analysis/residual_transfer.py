"""Does the residual model transfer across operator families?

The speed-of-light study fits T_measured ~ T_min + b1 stall_ms + b2
occupancy_deficit_ms. Raw milliseconds differ by orders of magnitude between
families, so a fit on one family can look transferable only because of scale.
Two questions, on the records of a study report:

* ``lofo_transfer``: leave each family out, fit on the rest, score R^2 on the
  held-out family, once on raw milliseconds and once on times normalised by
  T_min (so every family is on the "multiples of its roofline" scale);
* ``family_decodability``: can the family be told from the residual features
  alone (nearest-centroid, leave-one-out accuracy on the normalised
  features)? High decodability with low transfer means the families differ in
  kind, not only in scale.

``verdict`` combines them into one line. Reference parity:
kore/analysis/residual_transfer.py:46-267 (lofo transfer normalised and raw,
family decodability, verdict, render).
"""
from __future__ import annotations

import argparse
import json
from typing import Dict, List, Optional, Sequence

import numpy as np

from .study import Record


def _design(rs: Sequence[Record], normalized: bool):
    if normalized:
        X = np.array([[1.0, r.stall_ms / r.t_min_ms, r.occ_deficit_ms / r.t_min_ms] for r in rs])
        y = np.array([r.t_measured_ms / r.t_min_ms for r in rs])
    else:
        X = np.array([[r.t_min_ms, r.stall_ms, r.occ_deficit_ms, 1.0] for r in rs])
        y = np.array([r.t_measured_ms for r in rs])
    return X, y


def _r2(y: np.ndarray, pred: np.ndarray) -> Optional[float]:
    tot = float(((y - y.mean()) ** 2).sum())
    if tot <= 0:
        return None
    return 1.0 - float(((y - pred) ** 2).sum()) / tot


def lofo_transfer(rs: Sequence[Record], normalized: bool = True, min_train: int = 5,
                  min_test: int = 3) -> Dict[str, object]:
    rs = [r for r in rs if r.t_min_ms > 0]
    fams = sorted({r.family for r in rs})
    per: Dict[str, Optional[float]] = {}
    for f in fams:
        tr = [r for r in rs if r.family != f]
        te = [r for r in rs if r.family == f]
        if len(tr) < min_train or len(te) < min_test:
            continue
        Xtr, ytr = _design(tr, normalized)
        coef, *_ = np.linalg.lstsq(Xtr, ytr, rcond=None)
        Xte, yte = _design(te, normalized)
        per[f] = _r2(yte, Xte @ coef)
    vals = [v for v in per.values() if v is not None]
    return {"normalized": normalized, "per_family": per,
            "median_r2": float(np.median(vals)) if vals else None, "families": len(per)}


def family_decodability(rs: Sequence[Record]) -> Dict[str, object]:
    rs = [r for r in rs if r.t_min_ms > 0]
    fams = sorted({r.family for r in rs})
    if len(fams) < 2 or len(rs) < 4:
        return {"accuracy": None, "chance": None}
    X, _ = _design(rs, True)
    X = X[:, 1:]
    y = np.array([fams.index(r.family) for r in rs])
    correct = 0
    for i in range(len(rs)):
        mask = np.arange(len(rs)) != i
        cents = []
        for k in range(len(fams)):
            sel = mask & (y == k)
            cents.append(X[sel].mean(0) if sel.any() else np.full(X.shape[1], np.inf))
        d = [float(np.linalg.norm(X[i] - c)) for c in cents]
        correct += int(int(np.argmin(d)) == y[i])
    counts = np.bincount(y)
    return {"accuracy": correct / len(rs), "chance": float(counts.max() / counts.sum())}


def verdict(norm: Dict[str, object], decode: Dict[str, object]) -> str:
    r2 = norm.get("median_r2")
    acc, chance = decode.get("accuracy"), decode.get("chance")
    if r2 is None:
        return "UNDETERMINED: too few families with enough records"
    if r2 >= 0.5:
        return "TRANSFERS: one residual model serves unseen families (normalised median R^2 %.2f)" % r2
    if acc is not None and chance is not None and acc > chance + 0.2:
        return ("FAMILY-SPECIFIC: residual features identify the family (%.0f%% vs %.0f%% chance); "
                "fit per family" % (100 * acc, 100 * chance))
    return "DOES NOT TRANSFER: normalised median R^2 %.2f and families not separable" % r2


def run(rs: Sequence[Record]) -> dict:
    norm, raw = lofo_transfer(rs, True), lofo_transfer(rs, False)
    dec = family_decodability(rs)
    return {"normalized": norm, "raw": raw, "decodability": dec, "verdict": verdict(norm, dec)}


def render(res: dict) -> str:
    lines = ["# Residual-model transfer across families", "", f"**{res['verdict']}**", "",
             "| held-out family | R^2 normalised | R^2 raw |", "|---|---|---|"]
    fams = sorted(set(res["normalized"]["per_family"]) | set(res["raw"]["per_family"]))
    for f in fams:
        a, b = res["normalized"]["per_family"].get(f), res["raw"]["per_family"].get(f)
        lines.append(f"| {f} | {'-' if a is None else f'{a:.2f}'} | {'-' if b is None else f'{b:.2f}'} |")
    d = res["decodability"]
    if d.get("accuracy") is not None:
        lines += ["", f"family decodability: {d['accuracy']:.2f} (chance {d['chance']:.2f})"]
    return "\n".join(lines) + "\n"


def records_from_report(path: str) -> List[Record]:
    """Records of a study report written by ``kore_b200.analysis.p0_runner``."""
    from .p0_runner import KernelMeasure, to_record
    with open(path) as f:
        rep = json.load(f)
    out = []
    for m in rep.get("measures", []):
        km = KernelMeasure(**{k: m[k] for k in KernelMeasure.__dataclass_fields__ if k in m})
        r = to_record(km)
        if r is not None:
            out.append(r)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore residual-transfer")
    ap.add_argument("report")
    a = ap.parse_args(argv)
    res = run(records_from_report(a.report))
    print(render(res))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
