"""Figures of a speed-of-light study report as standalone SVG files (no
plotting library needed).

    python -m kore_b200.analysis.plots p0.json --out figs/

From the report of :mod:`kore_b200.analysis.p0_runner` it writes:

* ``eta_vs_speedup.svg``: roofline attainment eta against the speedup over the
  vendor baseline, one point per measured kernel, coloured by family (check a);
* ``residual_fit.svg``: time predicted by the residual model against the
  measured time, with the y = x line (check b);
* ``eta_by_family.svg``: eta of every kernel, grouped by family.

Reference parity: kore/analysis/plots.py (study figures), drawn directly as SVG.
"""
from __future__ import annotations

import argparse
import json
import math
import os
from typing import Dict, List, Optional, Sequence, Tuple

_PALETTE = ["#1f77b4", "#d62728", "#2ca02c", "#ff7f0e", "#9467bd", "#8c564b", "#e377c2", "#17becf", "#7f7f7f",
            "#bcbd22"]


def _esc(s: str) -> str:
    return str(s).replace("&", "&amp;").replace("<", "&lt;").replace(">", "&gt;")


def scatter_svg(series: Dict[str, List[Tuple[float, float]]], *, title: str, xlabel: str, ylabel: str,
                logx: bool = False, logy: bool = False, diagonal: bool = False, w: int = 640, h: int = 440) -> str:
    """An SVG scatter plot of named point series with axes, ticks and a legend."""
    pts = [p for s in series.values() for p in s if all(math.isfinite(v) for v in p)]
    if logx:
        pts = [p for p in pts if p[0] > 0]
    if logy:
        pts = [p for p in pts if p[1] > 0]
    tx = (lambda v: math.log10(v)) if logx else (lambda v: v)
    ty = (lambda v: math.log10(v)) if logy else (lambda v: v)
    if pts:
        xs, ys = [tx(p[0]) for p in pts], [ty(p[1]) for p in pts]
        x0, x1, y0, y1 = min(xs), max(xs), min(ys), max(ys)
    else:
        x0, x1, y0, y1 = 0.0, 1.0, 0.0, 1.0
    if diagonal:
        x0 = y0 = min(x0, y0)
        x1 = y1 = max(x1, y1)
    padx, pady = (x1 - x0) * 0.05 or 0.5, (y1 - y0) * 0.05 or 0.5
    x0, x1, y0, y1 = x0 - padx, x1 + padx, y0 - pady, y1 + pady
    L, R, T, B = 70, 150, 40, 55
    X = lambda v: L + (tx(v) - x0) / (x1 - x0) * (w - L - R)            # noqa: E731
    Y = lambda v: h - B - (ty(v) - y0) / (y1 - y0) * (h - T - B)        # noqa: E731
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{w}" height="{h}" font-family="sans-serif" '
           f'font-size="11">', f'<rect width="{w}" height="{h}" fill="white"/>',
           f'<text x="{w / 2}" y="20" text-anchor="middle" font-size="14">{_esc(title)}</text>',
           f'<line x1="{L}" y1="{h - B}" x2="{w - R}" y2="{h - B}" stroke="black"/>',
           f'<line x1="{L}" y1="{T}" x2="{L}" y2="{h - B}" stroke="black"/>',
           f'<text x="{(L + w - R) / 2}" y="{h - 15}" text-anchor="middle">{_esc(xlabel)}</text>',
           f'<text x="18" y="{(T + h - B) / 2}" text-anchor="middle" transform="rotate(-90 18 '
           f'{(T + h - B) / 2})">{_esc(ylabel)}</text>']
    for i in range(6):
        vx = x0 + (x1 - x0) * i / 5
        vy = y0 + (y1 - y0) * i / 5
        lx = 10 ** vx if logx else vx
        ly = 10 ** vy if logy else vy
        px = L + (w - L - R) * i / 5
        py = h - B - (h - T - B) * i / 5
        out.append(f'<line x1="{px:.1f}" y1="{h - B}" x2="{px:.1f}" y2="{h - B + 4}" stroke="black"/>'
                   f'<text x="{px:.1f}" y="{h - B + 16}" text-anchor="middle">{lx:.3g}</text>')
        out.append(f'<line x1="{L - 4}" y1="{py:.1f}" x2="{L}" y2="{py:.1f}" stroke="black"/>'
                   f'<text x="{L - 6}" y="{py + 4:.1f}" text-anchor="end">{ly:.3g}</text>')
    if diagonal:
        a, b = (10 ** x0 if logx else x0), (10 ** x1 if logx else x1)
        out.append(f'<line x1="{X(a):.1f}" y1="{Y(a):.1f}" x2="{X(b):.1f}" y2="{Y(b):.1f}" stroke="#999" '
                   f'stroke-dasharray="4 3"/>')
    for k, (name, s) in enumerate(sorted(series.items())):
        col = _PALETTE[k % len(_PALETTE)]
        for x, y in s:
            if not (math.isfinite(x) and math.isfinite(y)) or (logx and x <= 0) or (logy and y <= 0):
                continue
            out.append(f'<circle cx="{X(x):.1f}" cy="{Y(y):.1f}" r="3.5" fill="{col}" fill-opacity="0.75"/>')
        ly = T + 14 * k
        out.append(f'<circle cx="{w - R + 14}" cy="{ly}" r="4" fill="{col}"/>'
                   f'<text x="{w - R + 22}" y="{ly + 4}">{_esc(name)[:18]}</text>')
    out.append("</svg>")
    return "\n".join(out)


def _rows(rep: dict) -> List[dict]:
    return [m for m in rep.get("measures", []) if m.get("eta") is not None and m.get("speedup") is not None]


def fig_eta_vs_speedup(rep: dict) -> str:
    series: Dict[str, List[Tuple[float, float]]] = {}
    for m in _rows(rep):
        series.setdefault(m["family"], []).append((m["eta"], m["speedup"]))
    a = (rep.get("checks") or {}).get("a", {})
    t = "eta vs speedup" + (f" (Spearman {a['spearman']:.2f})" if "spearman" in a else "")
    return scatter_svg(series, title=t, xlabel="roofline attainment eta", ylabel="speedup vs vendor",
                       logy=True)


def fig_residual_fit(rep: dict) -> str:
    from .p0_runner import KernelMeasure, to_record
    from .study import _design, ols_r2
    recs = []
    for m in rep.get("measures", []):
        km = KernelMeasure(**{k: m[k] for k in KernelMeasure.__dataclass_fields__ if k in m})
        r = to_record(km)
        if r is not None:
            recs.append(r)
    series: Dict[str, List[Tuple[float, float]]] = {}
    if len(recs) >= 3:
        X, y = _design(recs)
        coef, r2 = ols_r2(X, y)
        pred = X @ coef
        for r, p in zip(recs, pred):
            series.setdefault(r.family, []).append((float(p), r.t_measured_ms))
        title = f"residual model: predicted vs measured (R^2 {r2:.2f})"
    else:
        title = "residual model: too few records"
    return scatter_svg(series, title=title, xlabel="predicted ms", ylabel="measured ms", logx=True, logy=True,
                       diagonal=True)


def fig_eta_by_family(rep: dict) -> str:
    fams = sorted({m["family"] for m in _rows(rep)})
    series: Dict[str, List[Tuple[float, float]]] = {}
    for m in _rows(rep):
        series.setdefault(m["family"], []).append((fams.index(m["family"]) + 1.0, m["eta"]))
    return scatter_svg(series, title="eta by family", xlabel="family (index)", ylabel="eta")


def write_all(rep: dict, out_dir: str) -> List[str]:
    os.makedirs(out_dir, exist_ok=True)
    paths = []
    for name, fn in (("eta_vs_speedup.svg", fig_eta_vs_speedup), ("residual_fit.svg", fig_residual_fit),
                     ("eta_by_family.svg", fig_eta_by_family)):
        p = os.path.join(out_dir, name)
        with open(p, "w") as f:
            f.write(fn(rep))
        paths.append(p)
    return paths


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore study-plots")
    ap.add_argument("report")
    ap.add_argument("--out", default="figs")
    a = ap.parse_args(argv)
    with open(a.report) as f:
        rep = json.load(f)
    for p in write_all(rep, a.out):
        print(p)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
