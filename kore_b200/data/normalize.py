"""Bring training shards onto this repository's prompt / response contract,
including shards generated for another GPU.

Rows are rewritten in content only, deterministically and idempotently:

* a kernel-engineering system prompt (any earlier or foreign version) is
  replaced by the canonical ``SYSTEM_PROMPT`` (sm_100a);
* an assistant turn that carries a kernel is re-rendered as
  ``ANALYSIS / PROPOSED_CHANGE / FULL_KERNEL`` (``normalize_assistant``);
* DPO ``chosen`` / ``rejected`` completions that carry a kernel become the
  kernel-only ``FULL_KERNEL`` completion, keeping ``margin`` / ``weight`` /
  provenance fields;
* conversations without a kernel (general chat, code, math retention rows)
  and agentic tool trajectories are left untouched.

``foreign_gpu`` marks rows whose measured numbers (speedups, wall times) were
taken on another GPU: they get ``"requires_reverify": true`` and keep their
original ``gpu`` field, and their kernels are not edited, so
:mod:`kore_b200.data.reverify` can re-measure them on B200 before they train
anything.

    python -m kore_b200.data.normalize in.jsonl --out out.jsonl [--foreign-gpu]
    python -m kore_b200.data.normalize in.jsonl --in-place

Reference parity: kore/data/normalize.py (canonical contract applied offline
to SFT / DPO / raw records, margin preserved, non-kernel rows untouched) and
upgrade_v1.py (in-place upgrade with a backup).
"""
from __future__ import annotations

import argparse
import json
import re
import shutil
from pathlib import Path
from typing import List, Optional, Tuple

from ..policy.format import FULL_KERNEL, SYSTEM_PROMPT, normalize_assistant, parse_response, wrap_full_kernel

_KERNEL_SYS = re.compile(r"(kernel|triton|cuda|hip)", re.I)
_KERNEL_SYS2 = re.compile(r"(GPU|ANALYSIS|FULL_KERNEL|optimi[sz])", re.I)


def is_kernel_system(content: str) -> bool:
    return bool(content) and bool(_KERNEL_SYS.search(content)) and bool(_KERNEL_SYS2.search(content))


def _has_kernel(content: str) -> bool:
    return bool(parse_response(content or "")["kernel"])


def _is_agentic(messages: List[dict]) -> bool:
    return any(m.get("role") == "tool" or "<tool_call>" in (m.get("content") or "") for m in messages)


def normalize_messages(messages: List[dict]) -> Tuple[List[dict], bool]:
    """(messages, changed). Agentic trajectories and kernel-free chats are returned as is."""
    if not messages or _is_agentic(messages):
        return messages, False
    kernel_chat = any(m.get("role") == "assistant" and _has_kernel(m.get("content", "")) for m in messages) or \
        any(m.get("role") == "system" and is_kernel_system(m.get("content", "")) for m in messages)
    if not kernel_chat:
        return messages, False
    out, changed = [], False
    for m in messages:
        role, c = m.get("role"), m.get("content") or ""
        if role == "system" and is_kernel_system(c) and c != SYSTEM_PROMPT:
            m = dict(m, content=SYSTEM_PROMPT)
            changed = True
        elif role == "assistant" and _has_kernel(c):
            nc = normalize_assistant(c)
            if nc != c:
                m = dict(m, content=nc)
                changed = True
        out.append(m)
    return out, changed


def _kernel_only(content: str) -> str:
    k = parse_response(content or "")["kernel"]
    return wrap_full_kernel(k) if k else content


def normalize_dpo_row(row: dict) -> Tuple[dict, bool]:
    out = dict(row)
    changed = False
    if isinstance(out.get("prompt"), list):
        out["prompt"], ch = normalize_messages(out["prompt"])
        changed |= ch
    for key in ("chosen", "rejected"):
        v = out.get(key)
        if isinstance(v, str) and _has_kernel(v) and not v.startswith(FULL_KERNEL):
            out[key] = _kernel_only(v)
            changed = True
        elif isinstance(v, list) and v and isinstance(v[-1], dict) and _has_kernel(v[-1].get("content", "")):
            k = _kernel_only(v[-1]["content"])
            if k != v[-1]["content"]:
                out[key] = v[:-1] + [dict(v[-1], content=k)]
                changed = True
    prov = out.get("_provenance") or {}
    for k in ("margin", "weight", "anchor"):                  # lift the pair's margin to the top level
        if k not in out and k in prov:
            out[k] = prov[k]
            changed = True
    return out, changed


def normalize_row(row: dict, foreign_gpu: bool = False) -> Tuple[dict, bool]:
    """Any shard row: SFT ({"messages"}), DPO ({"prompt", "chosen", "rejected"}),
    or a raw datagen record (repair ``messages``, win ``trajectory``, groups)."""
    changed = False
    if "chosen" in row and "rejected" in row:
        out, changed = normalize_dpo_row(row)
    else:
        out = dict(row)
        for key in ("messages", "trajectory"):
            if isinstance(out.get(key), list):
                out[key], ch = normalize_messages(out[key])
                changed |= ch
    if foreign_gpu and not out.get("requires_reverify"):
        out["requires_reverify"] = True
        changed = True
    return out, changed


def normalize_file(in_path: str, out_path: Optional[str] = None, *, in_place: bool = False,
                   foreign_gpu: bool = False) -> dict:
    """Rewrite a JSONL shard; with ``in_place`` the original is kept as
    ``<file>.bak`` (once). Malformed lines are carried over unchanged."""
    src = Path(in_path)
    dst = src if in_place else Path(out_path or str(src) + ".normalized")
    rows, n_changed, n_bad = [], 0, 0
    for line in src.read_text().splitlines():
        if not line.strip():
            continue
        try:
            row = json.loads(line)
        except json.JSONDecodeError:
            rows.append(line)
            n_bad += 1
            continue
        new, ch = normalize_row(row, foreign_gpu)
        n_changed += int(ch)
        rows.append(json.dumps(new))
    if in_place:
        bak = Path(str(src) + ".bak")
        if not bak.exists():
            shutil.copyfile(src, bak)
    dst.parent.mkdir(parents=True, exist_ok=True)
    dst.write_text("\n".join(rows) + ("\n" if rows else ""))
    return {"rows": len(rows), "changed": n_changed, "malformed": n_bad, "out": str(dst)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore normalize")
    ap.add_argument("inputs", nargs="+")
    ap.add_argument("--out", default=None, help="output file (one input) or directory")
    ap.add_argument("--in-place", action="store_true")
    ap.add_argument("--foreign-gpu", action="store_true", help="rows measured on another GPU: mark for re-verify")
    a = ap.parse_args(argv)
    for p in a.inputs:
        out = None
        if a.out:
            out = str(Path(a.out) / Path(p).name) if (len(a.inputs) > 1 or Path(a.out).is_dir()) else a.out
        print(json.dumps(normalize_file(p, out, in_place=a.in_place, foreign_gpu=a.foreign_gpu)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
