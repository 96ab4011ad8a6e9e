"""Nsight Compute counter collection for candidate kernels (replaces the
reference's rocprofv3 PMC passes, kore/verifier/pmc.py:162-517).

``collect_counters`` re-runs the driver on the primary shape under
``ncu --clock-control none`` with a small metric list (few passes, one kernel
launch captured) and returns ``{metric: value}``; parsing is in
:func:`parse_ncu_csv`. Counters feed the white-box potential and the dense
profile reward. The capture is small by construction: one shape, ``-c 1``.
"""
from __future__ import annotations

import csv
import io
import os
import shutil
import subprocess
from typing import Dict, Optional

METRICS = [
    "gpu__time_duration.sum",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
    "launch__registers_per_thread",
]


def parse_ncu_csv(text: str) -> Dict[str, float]:
    """Parse ``ncu --csv`` (long format: one metric per row). When several
    kernels were captured, the last value of each metric wins."""
    out: Dict[str, float] = {}
    start = text.find('"ID"')
    if start < 0:
        return out
    for row in csv.DictReader(io.StringIO(text[start:])):
        name, val = row.get("Metric Name"), row.get("Metric Value")
        if not name or val is None:
            continue
        try:
            v = float(val.replace(",", ""))
        except ValueError:
            continue
        unit = (row.get("Metric Unit") or "").lower()
        scale = {"kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "usecond": 1e3, "msecond": 1e6}.get(unit, 1.0)
        out[name] = v * scale
    return out


def ncu_available() -> bool:
    return shutil.which("ncu") is not None


def collect_counters(env, kpath: str, work: str, kernel_regex: Optional[str] = None) -> Dict[str, float]:
    if not ncu_available():
        return {}
    prim = env.task.shape("primary") or env.task.shapes[0]
    cmd = ["ncu", "--clock-control", "none", "--csv", "--metrics", ",".join(METRICS), "-c", "1"]
    if kernel_regex:
        cmd += ["-k", f"regex:{kernel_regex}"]
    cmd += [env.python, "-m", "kore_b200.tasks.driver", "--task", env.task.task_id, "--kernel", kpath,
            "--shape", prim.name, "--trials", "5"]
    try:
        r = subprocess.run(cmd, cwd=work, capture_output=True, text=True, timeout=env.timeout,
                           env=env._env())
    except subprocess.TimeoutExpired:
        return {}
    return parse_ncu_csv(r.stdout)


def parse_ptxas(text: str) -> Dict[str, Dict[str, int]]:
    """``-Xptxas -v`` report -> {function: {registers, spill_stores, spill_loads, smem}}."""
    import re
    out: Dict[str, Dict[str, int]] = {}
    cur = None
    for line in text.splitlines():
        m = re.search(r"Function properties for (\S+)", line)
        if m:
            cur = m.group(1)
            out.setdefault(cur, {})
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and cur:
            out[cur]["spill_stores"], out[cur]["spill_loads"] = int(m.group(1)), int(m.group(2))
        m = re.search(r"Used (\d+) registers", line)
        if m and cur:
            out[cur]["registers"] = int(m.group(1))
            m2 = re.search(r"(\d+) bytes smem", line)
            if m2:
                out[cur]["smem"] = int(m2.group(1))
    return out
