"""Nsight Compute counters for candidate kernels on B200.

Named metric sets (``METRIC_SETS``) say what to ask ``ncu`` for; each set is
collected in one or more invocations (``metric_passes``) that stay small: a
handful of metrics from few hardware units, one captured launch (``-c 1``),
``--clock-control none``. Larger sets are split by hardware unit so no single
capture replays the kernel dozens of times, and the per-invocation results
are merged (their keys are disjoint).

``collect_counters`` runs the task driver on the primary shape under ncu for
every pass of a set and returns ``{metric: value}`` in base units. The pure
helpers turn those into the quantities the reward and the bottleneck analysis
reason about: DRAM bytes, L2 hit rate, tensor-pipe busy fraction, achieved
occupancy, issue activity and the top warp-stall reasons, with a one-line
diagnosis. ``counter`` tolerates the metric-name variants ncu prints
(``.avg`` / ``.sum`` and ``_active`` / ``_elapsed`` percent forms).

Reference parity: the reference's rocprofv3 counter sets, multi-pass
grounding collection and derived metrics (kore/verifier/pmc.py:162-517:
counter_passes, l2_hit_rate, hbm_bytes, est_occupancy, mfma_busy_fraction),
re-made for Nsight Compute metric names; the occupancy model is in
:mod:`kore_b200.verifier.occupancy`.
"""
from __future__ import annotations

import shutil
import subprocess
from typing import Dict, List, Optional, Tuple

from .parsers.ncu import STALL_PREFIX, STALL_SUFFIX, parse_ncu_long_csv
from .parsers.ptxas import parse_ptxas_report

_STALLS = ["long_scoreboard", "short_scoreboard", "wait", "barrier", "membar", "mio_throttle",
           "lg_throttle", "math_pipe_throttle", "tex_throttle", "no_instruction", "branch_resolving",
           "dispatch_stall", "drain", "sleeping", "misc", "not_selected", "selected"]

METRIC_SETS: Dict[str, List[List[str]]] = {
    # the default: time, DRAM, SM / tensor activity, occupancy, one stall, registers (one pass group)
    "standard": [[
        "gpu__time_duration.sum",
        "dram__bytes_read.sum",
        "dram__bytes_write.sum",
        "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
        "sm__throughput.avg.pct_of_peak_sustained_elapsed",
        "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
        "sm__warps_active.avg.pct_of_peak_sustained_active",
        "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
        "launch__registers_per_thread",
    ]],
    "memory": [[
        "gpu__time_duration.sum",
        "dram__bytes_read.sum",
        "dram__bytes_write.sum",
        "lts__t_sector_hit_rate.pct",
        "lts__t_bytes.sum",
        "l1tex__t_bytes.sum",
    ]],
    "compute": [[
        "gpu__time_duration.sum",
        "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
        "sm__inst_executed_pipe_fma.avg.pct_of_peak_sustained_active",
        "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
        "smsp__issue_active.avg.pct_of_peak_sustained_active",
    ]],
    # everything a bottleneck explanation needs, split by hardware unit
    "grounding": [
        ["gpu__time_duration.sum", "sm__cycles_active.avg", "sm__warps_active.avg.pct_of_peak_sustained_active",
         "smsp__issue_active.avg.pct_of_peak_sustained_active", "launch__registers_per_thread",
         "launch__occupancy_limit_registers", "launch__occupancy_limit_shared_mem",
         "launch__occupancy_limit_warps", "launch__occupancy_limit_blocks"],
        ["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
         "sm__inst_executed_pipe_fma.avg.pct_of_peak_sustained_active",
         "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
         "sm__inst_executed_pipe_lsu.avg.pct_of_peak_sustained_active"],
        ["dram__bytes_read.sum", "dram__bytes_write.sum",
         "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "lts__t_sector_hit_rate.pct",
         "lts__t_bytes.sum"],
        [STALL_PREFIX + s + STALL_SUFFIX for s in _STALLS],
    ],
}

# for callers of the earlier single-list API
METRICS = METRIC_SETS["standard"][0]


def metric_passes(name: str = "standard") -> List[List[str]]:
    """The ncu invocations (metric groups) that collect set ``name``."""
    if name not in METRIC_SETS:
        raise KeyError(f"unknown metric set {name!r}: {sorted(METRIC_SETS)}")
    return [list(g) for g in METRIC_SETS[name]]


def parse_ncu_csv(text: str) -> Dict[str, float]:
    """Parse ``ncu --csv`` (long format: one metric per row) into one dict in
    base units. When several kernels were captured, the last one's values win."""
    out: Dict[str, float] = {}
    for k in parse_ncu_long_csv(text):
        out.update(k.metrics)
    return out


def ncu_available() -> bool:
    return shutil.which("ncu") is not None


def ncu_command(metrics: List[str], target: List[str], kernel_regex: Optional[str] = None,
                skip: int = 0, nvtx_range: Optional[str] = None) -> List[str]:
    """One small capture: listed metrics, one launch, clocks left alone;
    ``nvtx_range`` restricts it to launches inside that NVTX push/pop range."""
    cmd = ["ncu", "--clock-control", "none", "--csv", "--metrics", ",".join(metrics), "-c", "1"]
    if nvtx_range:
        cmd += ["--nvtx", "--nvtx-include", f"{nvtx_range}/"]
    if skip:
        cmd += ["-s", str(int(skip))]
    if kernel_regex:
        cmd += ["-k", f"regex:{kernel_regex}"]
    return cmd + list(target)


def collect_counters(env, kpath: str, work: str, kernel_regex: Optional[str] = None,
                     metric_set: str = "standard", impl: str = "candidate") -> Dict[str, float]:
    """Counters of the first kernel launch of one call of the candidate (or,
    with ``impl="baseline"``, of the task's vendor baseline) on the task's
    primary shape, merged over the set's passes; {} without ncu or when a pass
    fails."""
    if not ncu_available():
        return {}
    prim = env.task.shape("primary") or env.task.shapes[0]
    target = [env.python, "-m", "kore_b200.tasks.driver", "--task", env.task.task_id, "--kernel", kpath,
              "--shape", prim.name, "--profile-run", impl]
    out: Dict[str, float] = {}
    for group in metric_passes(metric_set):
        try:
            r = subprocess.run(ncu_command(group, target, kernel_regex, nvtx_range="kore_profile"), cwd=work,
                               capture_output=True, text=True, timeout=env.timeout, env=env._env())
        except subprocess.TimeoutExpired:
            return out
        out.update(parse_ncu_csv(r.stdout))
    return out


def parse_ptxas(text: str) -> Dict[str, Dict[str, int]]:
    """``-Xptxas -v`` report -> {function: {registers, spill_stores, spill_loads, smem}}."""
    out: Dict[str, Dict[str, int]] = {}
    for name, ri in parse_ptxas_report(text).items():
        d = {"spill_stores": ri.spill_stores, "spill_loads": ri.spill_loads}
        if ri.registers:
            d["registers"] = ri.registers
            d["smem"] = ri.smem_bytes
        out[name] = d
    return out


# ------------------------------------------------------------------ derived metrics
def counter(c: Dict[str, float], *names: str) -> Optional[float]:
    """First present metric among ``names``; each name also matches its
    ``.sum``/``.avg`` and ``_active``/``_elapsed`` variants."""
    if not c:
        return None
    for n in names:
        for v in _variants(n):
            if v in c and c[v] is not None:
                try:
                    return float(c[v])
                except (TypeError, ValueError):
                    continue
    return None


def _variants(n: str) -> List[str]:
    out = [n]
    for a, b in ((".sum", ".avg"), (".avg", ".sum"), ("_sustained_active", "_sustained_elapsed"),
                 ("_sustained_elapsed", "_sustained_active")):
        if a in n:
            out.append(n.replace(a, b))
    return out


def dram_bytes(c: Dict[str, float]) -> Optional[float]:
    r = counter(c, "dram__bytes_read.sum")
    w = counter(c, "dram__bytes_write.sum")
    if r is None and w is None:
        return counter(c, "dram__bytes.sum")
    return (r or 0.0) + (w or 0.0)


def l2_hit_rate(c: Dict[str, float]) -> Optional[float]:
    v = counter(c, "lts__t_sector_hit_rate.pct")
    return None if v is None else max(0.0, min(1.0, v / 100.0))


def tensor_busy_fraction(c: Dict[str, float]) -> Optional[float]:
    v = counter(c, "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active")
    return None if v is None else max(0.0, min(1.0, v / 100.0))


def achieved_occupancy(c: Dict[str, float]) -> Optional[float]:
    v = counter(c, "sm__warps_active.avg.pct_of_peak_sustained_active")
    return None if v is None else max(0.0, min(1.0, v / 100.0))


def dram_throughput_fraction(c: Dict[str, float]) -> Optional[float]:
    v = counter(c, "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed")
    return None if v is None else max(0.0, min(1.0, v / 100.0))


def top_stalls(c: Dict[str, float], n: int = 3) -> List[Tuple[str, float]]:
    """Largest warp-stall reasons (cycles per issued instruction), excluding
    the scheduler's own selected / not-selected states."""
    s = {k[len(STALL_PREFIX):-len(STALL_SUFFIX)]: v for k, v in (c or {}).items()
         if k.startswith(STALL_PREFIX) and k.endswith(STALL_SUFFIX)}
    s = {k: v for k, v in s.items() if k not in ("selected", "not_selected")}
    return sorted(s.items(), key=lambda kv: -kv[1])[:n]


def achieved_bandwidth(c: Dict[str, float]) -> Optional[float]:
    """DRAM bytes per second over the captured launch."""
    b, t = dram_bytes(c), counter(c, "gpu__time_duration.sum")
    if b is None or not t:
        return None
    return b / (t * 1e-9)


def diagnose(c: Dict[str, float], flops: Optional[float] = None) -> str:
    """One-line limiter of one launch: tensor pipe, DRAM, latency (with the top
    stall) or occupancy; ``flops`` (the kernel's algorithmic FLOPs) lets the
    text say whether the tensor pipe should be the limiter at all."""
    tc, dr, occ = tensor_busy_fraction(c), dram_throughput_fraction(c), achieved_occupancy(c)
    stalls = top_stalls(c, 1)
    b = dram_bytes(c)
    if flops and b:
        intensity = flops / max(b, 1.0)
        kind = "compute-bound by intensity" if intensity > 300 else "memory-bound by intensity"
    else:
        kind = None
    if tc is not None and tc >= 0.7:
        msg = f"tensor pipe busy {tc:.0%}: at the tensor roofline"
    elif dr is not None and dr >= 0.7:
        msg = f"DRAM throughput {dr:.0%} of peak: memory-bound"
    elif occ is not None and occ < 0.15 and (tc is None or tc < 0.5):
        msg = f"achieved occupancy {occ:.0%}: too few warps to hide latency"
    else:
        parts = []
        if tc is not None:
            parts.append(f"tensor {tc:.0%}")
        if dr is not None:
            parts.append(f"DRAM {dr:.0%}")
        msg = "latency-bound (" + ", ".join(parts) + ")" if parts else "no counters"
        if stalls:
            msg += f", top stall {stalls[0][0]} ({stalls[0][1]:.2f} cycles/issue)"
    return f"{msg}; {kind}" if kind else msg
