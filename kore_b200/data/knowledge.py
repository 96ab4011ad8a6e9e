"""B200 optimisation knowledge and an experience ledger for data generation.

Two aids for the teacher model that writes kernels during datagen:

* :func:`live_system_prompt` adds the relevant sections of the B200 playbook
  (``knowledge/b200_playbook.md``: general rules plus the section of the
  task's operation class and the pitfalls) to the system prompt the teacher
  sees while generating. It is never written into a stored trajectory: the
  stored turns keep the canonical ``SYSTEM_PROMPT``, so the policy's
  train-time and deploy-time prompts stay identical.
* :class:`ExperienceLedger` turns failed and regressed attempts on a task
  into a short, deduplicated list of "do not repeat" constraints (what was
  changed against the parent kernel and what happened), which later turns
  and other trajectories of the same task see in their generation context.

Pure functions of their inputs (the playbook file is read once and cached).
Reference parity: kore/data/amd_knowledge.py (live system prompt and the
experience ledger), with a B200 playbook written for this repository.
"""
from __future__ import annotations

import functools
import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Sequence

PLAYBOOK_PATH = Path(__file__).resolve().parent / "knowledge" / "b200_playbook.md"
_ALWAYS = ("general", "pitfalls")
_FALLBACK = ("# B200 (sm_100a) kernel playbook\n\n## general\n"
             "- 148 SMs, 227 KB shared memory per block, 126 MB L2, ~6.5 TB/s HBM, tcgen05 tensor cores "
             "(no wgmma on sm_100a). 16-byte accesses, fp32 accumulation, fuse elementwise epilogues, size grids "
             "to multiples of 148 or go persistent.\n")


@functools.lru_cache(maxsize=1)
def playbook_sections() -> Dict[str, str]:
    """{section name: markdown body} of the playbook."""
    try:
        text = PLAYBOOK_PATH.read_text()
    except OSError:
        text = _FALLBACK
    out: Dict[str, str] = {}
    for m in re.finditer(r"^## (\w+)\n(.*?)(?=^## |\Z)", text, re.M | re.S):
        out[m.group(1)] = m.group(2).strip()
    return out


def sections_for(operation: Optional[str]) -> List[str]:
    from ..value.features import op_class
    oc = op_class(operation or "")
    alias = {"train": "elementwise", "sample": "reduce", "ssm": "reduce", "conv": "gemm", "other": "elementwise"}
    name = alias.get(oc, oc)
    secs = playbook_sections()
    order = ["general"] + ([name] if name in secs and name not in _ALWAYS else []) + ["pitfalls"]
    return [s for s in order if s in secs]


def live_system_prompt(base: str, task=None, operation: Optional[str] = None, max_chars: int = 6000) -> str:
    """``base`` plus the playbook sections for the task's operation, capped at
    ``max_chars`` of added text (whole bullet lines only)."""
    op = operation or (getattr(task, "operation", None) if task is not None else None)
    secs = playbook_sections()
    lines: List[str] = ["", "", "B200 optimisation notes (for this generation):"]
    used = 0
    for s in sections_for(op):
        head = f"[{s}]"
        body = [ln for ln in secs[s].splitlines() if ln.strip()]
        for ln in [head] + body:
            if used + len(ln) + 1 > max_chars:
                return base + "\n".join(lines)
            lines.append(ln)
            used += len(ln) + 1
    return base + "\n".join(lines)


@dataclass
class Attempt:
    outcome: str                       # compile_fail | incorrect | slower | timeout
    change: str                        # what differed from the parent kernel
    detail: str = ""


def describe_change(parent: str, child: str) -> str:
    """What the child changed against the parent, in schedule terms (tile
    sizes, warps, stages, tensor-core path, TMA, vector width, ...)."""
    from ..value.features import schedule_features, tensor_core_tier
    a, b = schedule_features(parent or ""), schedule_features(child or "")
    names = {"log2_block_m": "BLOCK_M", "log2_block_n": "BLOCK_N", "log2_block_k": "BLOCK_K",
             "log2_block": "BLOCK", "log2_num_warps": "num_warps", "log2_num_stages": "num_stages",
             "log2_group_size_m": "GROUP_SIZE_M", "log2_threads": "threads per block",
             "log2_max_tile": "tile size"}
    parts = []
    for k, n in names.items():
        if a.get(k) != b.get(k):
            va = int(round(2 ** a[k])) if a.get(k) else "unset"
            vb = int(round(2 ** b[k])) if b.get(k) else "unset"
            parts.append(f"{n} {va} -> {vb}")
    ta, tb = tensor_core_tier(parent or ""), tensor_core_tier(child or "")
    if ta != tb:
        parts.append(f"tensor-core path {ta} -> {tb}")
    for k, n in (("tl_dot", "tl.dot"), ("tma", "TMA loads"), ("vec16", "16-byte vectors"), ("atomics", "atomics"),
                 ("exp2", "exp2"), ("masked", "boundary masks"), ("fp32_acc", "fp32 accumulator"),
                 ("cluster", "thread-block clusters")):
        if a.get(k) != b.get(k):
            parts.append(("added " if b.get(k) else "removed ") + n)
    return "; ".join(parts) if parts else "a rewrite with the same schedule knobs"


def _short(text: str, n: int = 140) -> str:
    t = " ".join((text or "").split())
    m = re.search(r"(error[^.;]*|SNR[^.;]*|mismatch[^.;]*)", t, re.I)
    t = m.group(1) if m else t
    return t[:n]


@dataclass
class ExperienceLedger:
    """Failed / regressed attempts per task, distilled into constraints."""
    max_items: int = 8
    items: Dict[str, List[Attempt]] = field(default_factory=dict)

    def record(self, task_id: str, parent_src: str, child_src: str, *, compiled: bool, correct: bool,
               parent_ms: Optional[float] = None, child_ms: Optional[float] = None, error: str = "") -> bool:
        """Add one attempt when it failed or regressed; returns whether it was kept."""
        if not compiled:
            outcome, detail = "compile_fail", _short(error)
        elif not correct:
            outcome, detail = "incorrect", _short(error)
        elif parent_ms and child_ms and child_ms > parent_ms * 1.02:
            outcome, detail = "slower", f"{child_ms:.3f} ms vs {parent_ms:.3f} ms"
        else:
            return False
        att = Attempt(outcome, describe_change(parent_src, child_src), detail)
        lst = self.items.setdefault(task_id, [])
        if any(x.outcome == att.outcome and x.change == att.change for x in lst):
            return False
        lst.append(att)
        del lst[: max(0, len(lst) - self.max_items)]
        return True

    def constraints(self, task_id: str) -> List[str]:
        verbs = {"compile_fail": "did not compile", "incorrect": "gave wrong results", "slower": "was slower",
                 "timeout": "timed out"}
        out = []
        for a in self.items.get(task_id, []):
            s = f"- {a.change}: {verbs.get(a.outcome, a.outcome)}"
            if a.detail:
                s += f" ({a.detail})"
            out.append(s)
        return out

    def block(self, task_id: str) -> str:
        c = self.constraints(task_id)
        if not c:
            return ""
        return "Earlier attempts on this task (do not repeat them):\n" + "\n".join(c)


def generation_messages(stored: Sequence[dict], task=None, ledger: Optional[ExperienceLedger] = None,
                        task_id: Optional[str] = None) -> List[dict]:
    """The teacher's view of a stored conversation: the system prompt with the
    playbook added and, when a ledger has entries for the task, its
    constraints appended to the last user turn. ``stored`` is not modified."""
    msgs = [dict(m) for m in stored]
    if msgs and msgs[0].get("role") == "system":
        msgs[0]["content"] = live_system_prompt(msgs[0]["content"], task)
    tid = task_id or getattr(task, "task_id", None)
    if ledger is not None and tid:
        blk = ledger.block(tid)
        if blk:
            for m in reversed(msgs):
                if m.get("role") == "user":
                    m["content"] = m["content"] + "\n\n" + blk
                    break
    return msgs
