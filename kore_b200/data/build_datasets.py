"""Assemble training sets from factory records.

* SFT: repair records (chat messages) + wins (trajectories) + optional
  general replay rows; repair rows are tagged so the SFT loader up-weights them.
* DPO: preference pairs from ranked groups (chosen = faster correct kernel).
* RFT: rejection-sampled fine-tuning set = correct, fastest candidates.
Rows whose task is in the held-out split are dropped (leakage guard), then
near-duplicates and low-quality kernels are filtered; general-replay rows that
near-duplicate a prompt of the bundled retention evaluations are dropped. CLI:
``kore build-datasets {sft,dpo,rft} --inputs a.jsonl,b.jsonl --out out.jsonl``.
Reference parity: kore/data/build_datasets.py:124-686.
"""
from __future__ import annotations

import argparse
from typing import List, Optional, Sequence

from ..policy.format import SYSTEM_PROMPT, parse_response
from ..tasks.registry import split_tasks
from .datasets import write_jsonl
from .hygiene import dedup, quality_ok
from .schemas import RankedGroupRecord, RepairRecord, WinRecord, read_records


def _heldout(seed: int = 0) -> set:
    return set(split_tasks(seed)[1])


def eval_prompts() -> List[str]:
    """Prompts of the bundled retention-evaluation sets (no row of a training
    mix may near-duplicate one of them)."""
    import glob
    import json
    import os
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "eval", "data")
    out = []
    for p in sorted(glob.glob(os.path.join(root, "*.jsonl"))):
        with open(p) as f:
            for line in f:
                try:
                    d = json.loads(line)
                except json.JSONDecodeError:
                    continue
                for k in ("prompt", "question", "instruction", "turns"):
                    v = d.get(k)
                    if isinstance(v, list):
                        v = "\n".join(str(x) for x in v)
                    if isinstance(v, str) and len(v) >= 40:
                        out.append(v)
                        break
    return out


def _user_text(row: dict) -> str:
    return "\n".join(m.get("content", "") for m in row.get("messages", []) if m.get("role") == "user")


def build_sft(paths: Sequence[str], out: str, *, seed: int = 0, general: Optional[str] = None) -> int:
    held = _heldout(seed)
    rows = []
    for p in paths:
        for r in read_records(p):
            if r.task_id in held:
                continue
            if isinstance(r, RepairRecord):
                rows.append({"messages": r.messages, "_source": "repair", "task_id": r.task_id})
            elif isinstance(r, WinRecord):
                rows.append({"messages": r.trajectory, "_source": "win", "task_id": r.task_id})
    rows = [r for r in rows if quality_ok(parse_response(r["messages"][-1]["content"]).get("kernel", "")
                                          if r["messages"][-1]["role"] == "assistant" else "x = 0")]
    rows = dedup(rows, key=lambda r: r["messages"][-1]["content"])
    if general:
        from .datasets import read_jsonl
        from .hygiene import decontaminate
        # general replay rows must not contain the retention evaluations' prompts
        rows += decontaminate(read_jsonl(general), eval_prompts(), key=_user_text)
    write_jsonl(out, rows)
    return len(rows)


def build_dpo(paths: Sequence[str], out: str, *, seed: int = 0) -> int:
    held = _heldout(seed)
    rows = []
    for p in paths:
        for r in read_records(p, RankedGroupRecord):
            if r.task_id in held:
                continue
            for c, j in r.preferences:
                ch, rj = r.candidates[c], r.candidates[j]
                prompt = [{"role": "system", "content": SYSTEM_PROMPT},
                          {"role": "user", "content": f"Optimize task {r.task_id}."}]
                rows.append({"prompt": prompt, "chosen": [{"role": "assistant", "content": ch.get("response") or ch["source"]}],
                             "rejected": [{"role": "assistant", "content": rj.get("response") or rj["source"]}],
                             "task_id": r.task_id})
    write_jsonl(out, rows)
    return len(rows)


def build_rft(paths: Sequence[str], out: str, *, seed: int = 0, top: int = 1) -> int:
    held = _heldout(seed)
    rows = []
    for p in paths:
        for r in read_records(p, RankedGroupRecord):
            if r.task_id in held:
                continue
            good = sorted([c for c in r.candidates if c.get("correct")], key=lambda c: c.get("wall_us") or 1e30)
            for c in good[:top]:
                rows.append({"messages": [{"role": "system", "content": SYSTEM_PROMPT},
                                          {"role": "user", "content": f"Optimize task {r.task_id}."},
                                          {"role": "assistant", "content": c.get("response") or c["source"]}],
                             "_source": "rft", "task_id": r.task_id})
    write_jsonl(out, rows)
    return len(rows)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore build-datasets")
    ap.add_argument("kind", choices=["sft", "dpo", "rft"])
    ap.add_argument("--inputs", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--general", default=None)
    a = ap.parse_args(argv)
    paths = [p for p in a.inputs.split(",") if p]
    n = {"sft": lambda: build_sft(paths, a.out, general=a.general), "dpo": lambda: build_dpo(paths, a.out),
         "rft": lambda: build_rft(paths, a.out)}[a.kind]()
    print(f"[build-datasets] {a.kind}: {n} rows -> {a.out}")
    return 0
