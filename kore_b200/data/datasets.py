"""JSONL dataset loaders for the trainers (torch-free).

* SFT: chat rows ``{"messages": [...]}``; rows marked as repair
  (``_provenance.kind == "repair"`` or ``_source == "repair"``) are emitted
  ``round(repair_weight)`` times (reference: kore/policy/sft.py:180-215).
* DPO: ``{"prompt", "chosen", "rejected"}`` rows (strings or message lists),
  optional ``weight`` applied as multiplicity (kore/policy/dpo.py:207-234).
* Midtrain: ``{"text"}`` rows, or chat rows flattened to text; malformed
  lines are skipped (kore/policy/midtrain.py:38-78).
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Dict, List


def read_jsonl(path) -> List[dict]:
    rows = []
    for line in Path(path).read_text(encoding="utf-8", errors="replace").splitlines():
        line = line.strip()
        if not line:
            continue
        try:
            rows.append(json.loads(line))
        except json.JSONDecodeError:
            continue
    return rows


def write_jsonl(path, rows) -> None:
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")


def is_repair(rec: dict) -> bool:
    prov = rec.get("_provenance") or {}
    return prov.get("kind") == "repair" or rec.get("_source") == "repair"


def load_sft_rows(path, repair_weight: float = 1.0) -> List[Dict]:
    factor = max(1, int(round(repair_weight)))
    out = []
    for rec in read_jsonl(path):
        msgs = rec["messages"] if isinstance(rec, dict) and "messages" in rec else rec
        if not isinstance(msgs, list):
            continue
        out.append({"messages": msgs})
        if factor > 1 and isinstance(rec, dict) and is_repair(rec):
            out.extend({"messages": msgs} for _ in range(factor - 1))
    return out


def _as_messages(x, role: str) -> List[dict]:
    if isinstance(x, list):
        return x
    return [{"role": role, "content": str(x)}]


def load_dpo_rows(path) -> List[Dict]:
    out = []
    for rec in read_jsonl(path):
        if not all(k in rec for k in ("prompt", "chosen", "rejected")):
            continue
        row = {"prompt": _as_messages(rec["prompt"], "user"),
               "chosen": _as_messages(rec["chosen"], "assistant"),
               "rejected": _as_messages(rec["rejected"], "assistant")}
        w = rec.get("weight", 1)
        n = max(1, int(round(float(w)))) if isinstance(w, (int, float)) else 1
        out.extend(dict(row) for _ in range(n))
    return out


def load_text_rows(path) -> List[str]:
    out = []
    for rec in read_jsonl(path):
        if isinstance(rec, dict) and isinstance(rec.get("text"), str):
            t = rec["text"]
        elif isinstance(rec, dict) and isinstance(rec.get("messages"), list):
            t = "\n\n".join(f"{m.get('role', 'user')}: {m.get('content', '')}" for m in rec["messages"]
                            if str(m.get("content", "")).strip())
        elif isinstance(rec, str):
            t = rec
        else:
            continue
        t = t.strip()
        if t:
            out.append(t)
    return out
