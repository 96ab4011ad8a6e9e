"""ptxas ``-v`` reports and nvcc diagnostics.

``nvcc -Xptxas -v`` prints, per compiled entry, its stack frame and spill
bytes and a "Used N registers, used B barriers, S bytes smem, C bytes cmem[i]"
line; ``parse_ptxas_report`` turns those into :class:`RegisterInfo` records
keyed by the (mangled) entry name, and ``RegisterInfo.residency`` applies the
sm_100a occupancy model to them. ``parse_nvcc_diagnostics`` splits nvcc /
ptxas output into errors and warnings with file and line. Reference parity:
kore/verifier/parsers/compiler_output.py:10-125 (register info, spill flag,
occupancy analysis, error and warning lists) for the reference's compiler.
"""
from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

from ..occupancy import Occupancy, occupancy

_ENTRY = re.compile(r"(?:Compiling entry function|Function properties for) '?([^'\s]+)'?")
_SPILL = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")
_USED = re.compile(r"Used (\d+) registers")
_BARS = re.compile(r"used (\d+) barriers")
_SMEM = re.compile(r"(\d+) bytes smem")
_CMEM = re.compile(r"(\d+) bytes cmem\[(\d+)\]")
_DIAG = re.compile(r"^(?P<file>[^\s(:]+)\((?P<line>\d+)\): (?P<kind>error|warning)[^:]*: (?P<msg>.*)$")
_PTXAS_DIAG = re.compile(r"^ptxas (?P<kind>error|warning|fatal)\s*: (?P<msg>.*)$")


@dataclass
class RegisterInfo:
    function: str
    registers: int = 0
    stack_bytes: int = 0
    spill_stores: int = 0
    spill_loads: int = 0
    smem_bytes: int = 0
    barriers: int = 0
    cmem_bytes: int = 0

    @property
    def has_spill(self) -> bool:
        return self.spill_stores > 0 or self.spill_loads > 0

    def residency(self, threads: int, dynamic_smem: int = 0, tmem_columns: int = 0) -> Occupancy:
        """Resident blocks per SM at ``threads`` threads per block (static
        shared memory from the report plus ``dynamic_smem``)."""
        return occupancy(threads, self.registers, self.smem_bytes + dynamic_smem, tmem_columns)

    def summary(self, threads: Optional[int] = None) -> str:
        s = f"{self.function[:60]}: {self.registers} regs"
        if self.has_spill:
            s += f", SPILLS {self.spill_stores}/{self.spill_loads} B (stores/loads)"
        if self.smem_bytes:
            s += f", {self.smem_bytes} B static smem"
        if threads:
            o = self.residency(threads)
            s += f"; at {threads} threads: {o.blocks_per_sm} block(s)/SM ({o.limiter})"
        return s


def parse_ptxas_report(text: str) -> Dict[str, RegisterInfo]:
    out: Dict[str, RegisterInfo] = {}
    cur: Optional[RegisterInfo] = None
    for line in text.splitlines():
        m = _ENTRY.search(line)
        if m:
            name = m.group(1)
            cur = out.setdefault(name, RegisterInfo(name))
            continue
        if cur is None:
            continue
        m = _SPILL.search(line)
        if m:
            cur.stack_bytes, cur.spill_stores, cur.spill_loads = (int(g) for g in m.groups())
        m = _USED.search(line)
        if m:
            cur.registers = int(m.group(1))
            b = _BARS.search(line)
            cur.barriers = int(b.group(1)) if b else 0
            sm = _SMEM.search(line)
            cur.smem_bytes = int(sm.group(1)) if sm else 0
            cur.cmem_bytes = sum(int(c.group(1)) for c in _CMEM.finditer(line))
    return out


def parse_nvcc_diagnostics(text: str) -> Tuple[List[dict], List[dict]]:
    """(errors, warnings); each {"file", "line", "message"} (file/line None for ptxas)."""
    errors: List[dict] = []
    warnings: List[dict] = []
    for line in text.splitlines():
        line = line.rstrip()
        m = _DIAG.match(line)
        if m:
            rec = {"file": m.group("file"), "line": int(m.group("line")), "message": m.group("msg")}
            (errors if m.group("kind") == "error" else warnings).append(rec)
            continue
        m = _PTXAS_DIAG.match(line)
        if m:
            rec = {"file": None, "line": None, "message": m.group("msg")}
            (warnings if m.group("kind") == "warning" else errors).append(rec)
    return errors, warnings
