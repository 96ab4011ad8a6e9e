"""Speed-of-light study runner: measures candidate kernels of real tasks and
feeds :mod:`kore_b200.analysis.study`'s three checks.

    python -m kore_b200.analysis.p0_runner --tasks rmsnorm_bf16,gemm_bf16 --kernels 6 --out p0.json
    python -m kore_b200.analysis.p0_runner --replay groups.jsonl --out p0.json     # no GPU needed

For each task it builds a small trajectory of sources (the task's seed plus
correctness-preserving variants from the transform library), and for each
source and shape runs the task driver in a child process: correctness first
(SNR against the fp32 oracle), then the alternating candidate / vendor bench
(median of repeated runs), then, when ``--pmc`` is given and ncu exists, one
small counter capture. A measured kernel becomes a
:class:`~kore_b200.analysis.study.Record`: eta = T_min / T_measured from the
roofline of the task's operation at that shape and the measured peaks, the
speedup over the vendor baseline, and the stall and occupancy-deficit
milliseconds of the residual decomposition (from the counters: the
long-scoreboard share of issue stalls and the missing fraction of achieved
occupancy, each times the time above the roofline).

``--replay`` mines already-measured candidates (ranked-group records with
wall times) instead of running anything. ``decide`` turns the three checks
into a go / no-go line; ``render`` prints a markdown report.

Reference parity: kore/analysis/p0_sol.py:141-802 (measure_kernel,
trajectory_sources, check_a/b/c, bootstrap CIs, decide, replay mining,
render), written for this repository's driver contract and ncu counters.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
from dataclasses import asdict, dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

from .rooflines import flops_bytes, resolve_peaks, peak_flops
from .study import Record, leave_one_family_out, p0_checks

_SNR = re.compile(r"SNR:\s*(-?[\d.]+)")
_CAND = re.compile(r"^CAND (\S+) ([\d.]+) ([\d.]+)", re.M)
_REF = re.compile(r"^REF (\S+) ([\d.]+) ([\d.]+)", re.M)


@dataclass
class KernelMeasure:
    task_id: str
    family: str
    label: str
    shape: str
    correct: bool
    snr_db: Optional[float] = None
    cand_ms: Optional[float] = None
    ref_ms: Optional[float] = None
    t_min_ms: Optional[float] = None
    counters: Dict[str, float] = field(default_factory=dict)
    error: str = ""

    @property
    def eta(self) -> Optional[float]:
        if self.cand_ms and self.t_min_ms:
            return self.t_min_ms / self.cand_ms
        return None

    @property
    def speedup(self) -> Optional[float]:
        if self.cand_ms and self.ref_ms:
            return self.ref_ms / self.cand_ms
        return None


def t_min_ms(operation: str, dims: Dict[str, int], dtype: str, peaks: Dict[str, float]) -> Optional[float]:
    fb = flops_bytes(operation, dims, dtype)
    if fb is None:
        return None
    f, b = fb
    return max(f / peak_flops(peaks, dtype), b / peaks["hbm_bytes_per_s"]) * 1e3


def decompose(counters: Dict[str, float], cand_ms: float, t_min: float) -> Tuple[float, float]:
    """(stall_ms, occupancy_deficit_ms): the time above the roofline split by
    the long-scoreboard share of issue stalls and by the missing fraction of
    achieved occupancy."""
    from ..verifier.pmc import achieved_occupancy, top_stalls
    excess = max(0.0, cand_ms - t_min)
    st = dict(top_stalls(counters, 32))
    tot = sum(st.values())
    stall_frac = (st.get("long_scoreboard", 0.0) / tot) if tot else 0.0
    occ = achieved_occupancy(counters)
    deficit = (1.0 - occ) if occ is not None else 0.0
    return excess * stall_frac, excess * deficit


def to_record(m: KernelMeasure) -> Optional[Record]:
    if not m.correct or m.eta is None or m.speedup is None:
        return None
    st, oc = decompose(m.counters, m.cand_ms, m.t_min_ms) if m.counters else (0.0, 0.0)
    return Record(m.task_id, m.family, m.eta, m.speedup, m.cand_ms, m.t_min_ms, st, oc)


# ------------------------------------------------------------------ measuring
def _run(cmd: List[str], cwd: str, timeout: int) -> Tuple[int, str]:
    try:
        r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True, timeout=timeout)
        return r.returncode, r.stdout + r.stderr
    except subprocess.TimeoutExpired:
        return -9, "TIMEOUT"


def measure_kernel(task, label: str, source: str, shape, peaks: Dict[str, float], *, snr_min: float = 20.0,
                   repeats: int = 3, pmc: bool = False, timeout: int = 300,
                   runner: Callable[[List[str], str, int], Tuple[int, str]] = _run) -> KernelMeasure:
    """Correctness, repeated bench and (optionally) counters of one source at one shape."""
    m = KernelMeasure(task.task_id, task.family, label, shape.name, False,
                      t_min_ms=t_min_ms(task.operation, shape.dims, task.dtype, peaks))
    with tempfile.TemporaryDirectory() as work:
        kp = os.path.join(work, "kernel.py")
        with open(kp, "w") as f:
            f.write(source)
        base = [sys.executable, "-m", "kore_b200.tasks.driver", "--task", task.task_id, "--kernel", kp]
        rc, out = runner(base + ["--shape", shape.name], work, timeout)
        snr = _SNR.findall(out)
        m.snr_db = float(snr[-1]) if snr else None
        m.correct = rc == 0 and m.snr_db is not None and m.snr_db >= snr_min
        if not m.correct:
            m.error = out[-400:]
            return m
        cands, refs = [], []
        for _ in range(max(1, repeats)):
            rc, out = runner(base + ["--bench-both", "--shapes", shape.name], work, timeout)
            c, r = _CAND.findall(out), _REF.findall(out)
            if rc == 0 and c and r:
                cands.append(float(c[-1][1]))
                refs.append(float(r[-1][1]))
        if cands:
            cands.sort()
            refs.sort()
            m.cand_ms, m.ref_ms = cands[len(cands) // 2], refs[len(refs) // 2]
        if pmc:
            from ..verifier.pmc import METRIC_SETS, ncu_available, ncu_command, parse_ncu_csv
            if ncu_available():
                for group in METRIC_SETS["grounding"]:
                    rc, out = runner(ncu_command(group, base + ["--shape", shape.name, "--profile-run", "candidate"],
                                                 nvtx_range="kore_profile"), work, timeout)
                    m.counters.update(parse_ncu_csv(out))
    return m


def trajectory_sources(task, max_kernels: int = 6) -> List[Tuple[str, str]]:
    """(label, source): the seed, then variants the transform library can
    apply to it (each a correctness-preserving rewrite), up to ``max_kernels``."""
    out = [("seed", task.seed_src)]
    try:
        from ..transform.calculus import admissible_actions
        seen = {task.seed_src}
        for a in admissible_actions(task.seed_src):
            if len(out) >= max_kernels:
                break
            if a.kind != "exact":                 # approximate rewrites change the result: not a study point
                continue
            src = a.apply(task.seed_src)
            if src and src not in seen:
                seen.add(src)
                out.append((a.name, src))
    except Exception:  # noqa: BLE001 - variants are optional
        pass
    return out[:max_kernels]


def mine_replay(paths: Sequence[str], peaks: Dict[str, float]) -> List[KernelMeasure]:
    """KernelMeasures from ranked-group records: each correct candidate with a
    wall time, against the parent's wall time as the baseline."""
    from ..data.schemas import RankedGroupRecord, read_records
    from ..tasks.registry import get_task
    out = []
    for p in paths:
        for r in read_records(p, RankedGroupRecord):
            try:
                t = get_task(r.task_id)
            except KeyError:
                continue
            sh = (t.shape(r.shape) if r.shape else None) or t.shape("primary") or t.shapes[0]
            tm = t_min_ms(t.operation, sh.dims, t.dtype, peaks)
            for i, c in enumerate(r.candidates):
                w = c.get("wall_us")
                ok = bool(c.get("correct")) and w
                out.append(KernelMeasure(t.task_id, t.family, f"cand{i}", sh.name, bool(ok), c.get("snr_db"),
                                         w / 1e3 if ok else None,
                                         r.parent_wall_us / 1e3 if r.parent_wall_us else None, tm,
                                         dict(c.get("counters") or {})))
    return out


# ------------------------------------------------------------------ verdicts
def decide(checks: Dict[str, dict]) -> str:
    v = [checks[k]["verdict"] for k in ("a", "b", "c")]
    if all(x == "PASS" for x in v):
        return "GO: roofline attainment ranks kernels and the residual model explains time"
    if "FAIL" in v[:2]:
        return "NO-GO: " + ("eta does not rank kernels" if v[0] == "FAIL" else "the residual model does not fit")
    return "CONDITIONAL: " + ", ".join(f"check {k} {x}" for k, x in zip("abc", v) if x != "PASS")


def run(measures: Sequence[KernelMeasure], iters: int = 1000) -> dict:
    recs = [r for r in (to_record(m) for m in measures) if r is not None]
    rep = {"n_measured": len(measures), "n_records": len(recs),
           "measures": [dict(asdict(m), eta=m.eta, speedup=m.speedup) for m in measures]}
    if len(recs) >= 4:
        checks = p0_checks(recs, iters=iters)
        rep["checks"] = checks
        rep["decision"] = decide(checks)
        rep["lofo_r2"] = leave_one_family_out(recs)
    else:
        rep["decision"] = "INSUFFICIENT: fewer than 4 correct, timed kernels"
    return rep


def render(rep: dict) -> str:
    lines = ["# Speed-of-light study", "", f"kernels measured: {rep['n_measured']}, usable records: "
             f"{rep['n_records']}", "", f"**{rep['decision']}**", ""]
    ch = rep.get("checks")
    if ch:
        lines += ["| check | value | 95% CI | verdict |", "|---|---|---|---|"]
        for k, name, key in (("a", "Spearman(eta, speedup)", "spearman"), ("b", "residual R^2", "r2"),
                             ("c", "monotone-in-valley", "monotone_frac")):
            c = ch[k]
            lines.append(f"| ({k}) {name} | {c[key]:.3f} | [{c['ci'][0]:.3f}, {c['ci'][1]:.3f}] | {c['verdict']} |")
    lofo = rep.get("lofo_r2") or {}
    if lofo:
        lines += ["", "Leave-one-family-out residual R^2: " + ", ".join(f"{k} {v:.2f}" for k, v in sorted(lofo.items()))]
    rows = [m for m in rep["measures"] if m.get("eta") is not None]
    if rows:
        lines += ["", "| task | kernel | shape | eta | speedup |", "|---|---|---|---|---|"]
        for m in rows[:50]:
            lines.append(f"| {m['task_id']} | {m['label']} | {m['shape']} | {m['eta']:.3f} | {m['speedup']:.2f} |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore study")
    ap.add_argument("--tasks", default="")
    ap.add_argument("--kernels", type=int, default=6)
    ap.add_argument("--shapes", type=int, default=1, help="bench shapes per task")
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--pmc", action="store_true")
    ap.add_argument("--replay", default="", help="ranked-group JSONL files instead of running kernels")
    ap.add_argument("--iters", type=int, default=1000, help="bootstrap resamples")
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    peaks = resolve_peaks()
    if a.replay:
        ms = mine_replay([p for p in a.replay.split(",") if p], peaks)
    else:
        from ..tasks.registry import get_task
        ms = []
        for tid in [t for t in a.tasks.split(",") if t]:
            t = get_task(tid)
            shapes = (t.bench_shapes() or t.shapes)[: a.shapes]
            for label, src in trajectory_sources(t, a.kernels):
                for sh in shapes:
                    ms.append(measure_kernel(t, label, src, sh, peaks, repeats=a.repeats, pmc=a.pmc))
    rep = run(ms, a.iters)
    with open(a.out, "w") as f:
        json.dump(rep, f, indent=1, default=str)
    with open(os.path.splitext(a.out)[0] + ".md", "w") as f:
        f.write(render(rep))
    print(rep["decision"])
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
