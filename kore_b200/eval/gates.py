"""Stage gates and the retention suite.

``retention_gate(base_scores, new_scores, epsilon)`` fails a stage when any
general-capability benchmark regresses by more than epsilon (absolute),
optionally requiring a significant kernel-skill gain. ``run_retention_suite``
scores a generation callable on local JSONL suites (each row
``{"prompt", "answer"}`` or ``{"prompt", "tests"}``); with no network, the
suites are whatever is provided locally, and results are cached per
(model, suite). Reference parity: kore/eval/gates.py:81-292,
kore/eval/retention.py.
"""
from __future__ import annotations

import json
import os
import re
from dataclasses import dataclass
from typing import Callable, Dict, Optional


@dataclass
class GateResult:
    passed: bool
    regressions: Dict[str, float]
    detail: str


def retention_gate(base: Dict[str, float], new: Dict[str, float], epsilon: float = 0.005) -> GateResult:
    regs = {k: base[k] - new.get(k, 0.0) for k in base if base[k] - new.get(k, 0.0) > epsilon}
    return GateResult(not regs, regs, "ok" if not regs else f"regressed beyond {epsilon}: {sorted(regs)}")


def kernel_gate(fastp_base: float, fastp_new: float, min_gain: float = 0.0) -> GateResult:
    ok = fastp_new >= fastp_base + min_gain
    return GateResult(ok, {} if ok else {"fast_p": fastp_base - fastp_new}, f"fast_p {fastp_base:.3f} -> {fastp_new:.3f}")


def _norm(s: str) -> str:
    return re.sub(r"\s+", " ", (s or "").strip().lower())


def score_row(row: dict, out: str) -> float:
    if "answer" in row:
        return float(_norm(str(row["answer"])) in _norm(out))
    if "tests" in row:
        ns: dict = {}
        code = re.search(r"```(?:python)?\n(.*?)```", out, re.DOTALL)
        try:
            exec((code.group(1) if code else out) + "\n" + row["tests"], ns)  # noqa: S102 - sandboxed by caller
            return 1.0
        except Exception:  # noqa: BLE001
            return 0.0
    return 0.0


def run_retention_suite(generate: Callable[[str], str], suites: Dict[str, str], cache_path: Optional[str] = None,
                        model_key: str = "model") -> Dict[str, float]:
    cache = {}
    if cache_path and os.path.exists(cache_path):
        cache = json.load(open(cache_path))
    out = {}
    for name, path in suites.items():
        key = f"{model_key}::{name}"
        if key in cache:
            out[name] = cache[key]
            continue
        rows = [json.loads(l) for l in open(path) if l.strip()]
        out[name] = sum(score_row(r, generate(r["prompt"])) for r in rows) / max(1, len(rows))
        cache[key] = out[name]
    if cache_path:
        json.dump(cache, open(cache_path, "w"))
    return out
