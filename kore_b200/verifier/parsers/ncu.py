"""Nsight Compute CSV exports -> per-kernel counter records.

Two layouts are read:

* the long layout of ``ncu --csv --metrics ...`` (one row per kernel and
  metric, columns "ID", "Kernel Name", "Block Size", "Grid Size",
  "Metric Name", "Metric Unit", "Metric Value");
* the wide layout of ``ncu -i report.ncu-rep --page raw --csv`` (a header row
  of metric names, a row of units, then one row per captured kernel).

Values are normalised to base units: bytes, nanoseconds, percent as printed,
plain counts. Reference parity: the reference's rocprofv3 CSV parser
(kore/verifier/parsers/rocprofv3.py:24-252, per-kernel PMC records with a
diagnosis); the counters are Nsight Compute's.
"""
from __future__ import annotations

import csv
import io
import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

_BYTES = {"byte": 1.0, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "tbyte": 1e12,
          "kibyte": 1024.0, "mibyte": 1024.0 ** 2, "gibyte": 1024.0 ** 3}
_TIME = {"nsecond": 1.0, "usecond": 1e3, "msecond": 1e6, "second": 1e9}
_RATE = {"byte/second": 1.0, "kbyte/second": 1e3, "mbyte/second": 1e6, "gbyte/second": 1e9,
         "tbyte/second": 1e12}
_FREQ = {"hz": 1.0, "khz": 1e3, "mhz": 1e6, "ghz": 1e9}

STALL_PREFIX = "smsp__average_warps_issue_stalled_"
STALL_SUFFIX = "_per_issue_active.ratio"


def _scale(unit: str) -> float:
    u = (unit or "").strip().lower()
    for table in (_BYTES, _TIME, _RATE, _FREQ):
        if u in table:
            return table[u]
    return 1.0


def _num(text: str) -> Optional[float]:
    t = (text or "").strip().replace(",", "")
    if not t or t.lower() in ("n/a", "nan", "-"):
        return None
    try:
        return float(t)
    except ValueError:
        return None


def _dims(text: str) -> Tuple[int, int, int]:
    nums = [int(x) for x in re.findall(r"\d+", text or "")]
    nums += [1] * (3 - len(nums))
    return nums[0], nums[1], nums[2]


@dataclass
class KernelCounters:
    """One captured kernel launch."""
    kernel: str
    launch_id: str = ""
    block: Tuple[int, int, int] = (1, 1, 1)
    grid: Tuple[int, int, int] = (1, 1, 1)
    metrics: Dict[str, float] = field(default_factory=dict)

    def get(self, *names: str) -> Optional[float]:
        for n in names:
            if n in self.metrics:
                return self.metrics[n]
        return None

    @property
    def threads_per_block(self) -> int:
        return self.block[0] * self.block[1] * self.block[2]

    @property
    def blocks(self) -> int:
        return self.grid[0] * self.grid[1] * self.grid[2]

    @property
    def duration_ns(self) -> Optional[float]:
        return self.get("gpu__time_duration.sum", "gpu__time_duration.avg")

    @property
    def dram_bytes(self) -> Optional[float]:
        r, w = self.get("dram__bytes_read.sum"), self.get("dram__bytes_write.sum")
        if r is None and w is None:
            return self.get("dram__bytes.sum")
        return (r or 0.0) + (w or 0.0)

    def stalls(self) -> Dict[str, float]:
        """Warp stall reasons (cycles per issued instruction), by short name."""
        out = {}
        for k, v in self.metrics.items():
            if k.startswith(STALL_PREFIX) and k.endswith(STALL_SUFFIX):
                out[k[len(STALL_PREFIX):-len(STALL_SUFFIX)]] = v
        return out

    def top_stalls(self, n: int = 3) -> List[Tuple[str, float]]:
        s = {k: v for k, v in self.stalls().items() if k not in ("selected", "not_selected")}
        return sorted(s.items(), key=lambda kv: -kv[1])[:n]

    def summary(self) -> str:
        parts = [self.kernel[:60]]
        d = self.duration_ns
        if d is not None:
            parts.append(f"{d / 1e3:.1f} us")
        b = self.dram_bytes
        if b is not None and d:
            parts.append(f"DRAM {b / 1e6:.1f} MB ({b / d:.0f} GB/s)")
        t = self.get("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
                     "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed")
        if t is not None:
            parts.append(f"tensor {t:.1f}%")
        top = self.top_stalls(2)
        if top:
            parts.append("stalls " + ", ".join(f"{k} {v:.2f}" for k, v in top))
        return "; ".join(parts)


def parse_ncu_long_csv(text: str) -> List[KernelCounters]:
    """``ncu --csv --metrics ...`` output (any log lines before the table are skipped)."""
    start = text.find('"ID"')
    if start < 0:
        return []
    kernels: Dict[str, KernelCounters] = {}
    order: List[str] = []
    for row in csv.DictReader(io.StringIO(text[start:])):
        kid = row.get("ID", "")
        if kid not in kernels:
            kernels[kid] = KernelCounters(row.get("Kernel Name", ""), kid, _dims(row.get("Block Size", "")),
                                          _dims(row.get("Grid Size", "")))
            order.append(kid)
        name = row.get("Metric Name")
        v = _num(row.get("Metric Value", ""))
        if name and v is not None:
            kernels[kid].metrics[name] = v * _scale(row.get("Metric Unit", ""))
    return [kernels[k] for k in order]


def parse_ncu_raw_csv(text: str) -> List[KernelCounters]:
    """``ncu -i <report> --page raw --csv``: header, units, one row per kernel."""
    start = text.find('"ID"')
    if start < 0:
        return []
    rows = list(csv.reader(io.StringIO(text[start:])))
    if len(rows) < 2:
        return []
    head = rows[0]
    units = rows[1] if len(rows) > 1 and not _looks_like_data(rows[1]) else [""] * len(head)
    body = rows[2:] if units is rows[1] else rows[1:]
    col = {h: i for i, h in enumerate(head)}
    out = []
    for r in body:
        if len(r) != len(head):
            continue
        kc = KernelCounters(r[col["Kernel Name"]] if "Kernel Name" in col else "", r[col["ID"]],
                            _dims(r[col["Block Size"]]) if "Block Size" in col else (1, 1, 1),
                            _dims(r[col["Grid Size"]]) if "Grid Size" in col else (1, 1, 1))
        for i, h in enumerate(head):
            if "__" not in h:           # metric names have a unit__counter form
                continue
            v = _num(r[i])
            if v is not None:
                kc.metrics[h] = v * _scale(units[i] if i < len(units) else "")
        out.append(kc)
    return out


def _looks_like_data(row: List[str]) -> bool:
    return bool(row) and row[0].strip().isdigit()
