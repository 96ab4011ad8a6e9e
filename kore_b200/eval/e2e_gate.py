"""End-to-end serving gate: does a trained checkpoint still serve as well as
its base?

A *workload* is a list of prompts (optionally with expected answers). The gate
serves it through a generation backend, measures

* throughput: generated tokens per second over the whole workload (wall clock
  of the backend call, which includes its batching), and
* accuracy: the fraction of answered prompts whose answer contains the
  expected one,

for the candidate and for the baseline checkpoint, and fails when throughput
drops by more than ``max_tput_drop`` or accuracy by more than ``max_acc_drop``.

Backends: this package's paged rollout engine (``engine_backend``), or any
OpenAI-compatible HTTP endpoint such as a vLLM or SGLang server
(``openai_backend``; used only when a URL is given, nothing is contacted
otherwise). A backend is ``generate(prompts) -> list of (text, n_tokens)``.

Reference behaviour: kore/eval/e2e_sglang_vllm.py:68-324.
"""
from __future__ import annotations

import json
import time
import urllib.request
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple

Backend = Callable[[List[str]], List[Tuple[str, int]]]


@dataclass
class Workload:
    prompts: List[str]
    answers: Optional[List[Optional[str]]] = None
    max_new_tokens: int = 256
    name: str = "workload"


@dataclass
class E2EResult:
    tokens_per_s: float
    accuracy: Optional[float]
    n: int
    seconds: float
    outputs: List[str] = field(default_factory=list)


def run_workload(backend: Backend, wl: Workload) -> E2EResult:
    t0 = time.perf_counter()
    outs = backend(list(wl.prompts))
    dt = max(time.perf_counter() - t0, 1e-9)
    texts = [o[0] for o in outs]
    ntok = sum(o[1] for o in outs)
    acc = None
    if wl.answers:
        graded = [(t, a) for t, a in zip(texts, wl.answers) if a is not None]
        acc = sum(str(a).strip().lower() in t.lower() for t, a in graded) / max(1, len(graded))
    return E2EResult(ntok / dt, acc, len(texts), dt, texts)


@dataclass
class GateVerdict:
    passed: bool
    candidate: E2EResult
    baseline: E2EResult
    detail: str


def e2e_gate(candidate: Backend, baseline: Backend, wl: Workload, *, max_tput_drop: float = 0.10,
             max_acc_drop: float = 0.02) -> GateVerdict:
    base = run_workload(baseline, wl)
    cand = run_workload(candidate, wl)
    reasons = []
    if cand.tokens_per_s < (1.0 - max_tput_drop) * base.tokens_per_s:
        reasons.append(f"throughput {cand.tokens_per_s:.1f} < {(1 - max_tput_drop):.2f} x {base.tokens_per_s:.1f}")
    if base.accuracy is not None and cand.accuracy is not None and cand.accuracy < base.accuracy - max_acc_drop:
        reasons.append(f"accuracy {cand.accuracy:.3f} < {base.accuracy:.3f} - {max_acc_drop}")
    return GateVerdict(not reasons, cand, base, "; ".join(reasons) or "ok")


def engine_backend(weights, tokenizer, *, max_new_tokens: int = 256, temperature: float = 0.0,
                   eos_ids: Sequence[int] = (), **engine_kw) -> Backend:
    """Serve through the paged rollout engine (continuous batching)."""
    from ..data.tokenizer import render_chat
    from ..engine.rollout import GenRequest, RolloutEngine
    eng = RolloutEngine(weights, **engine_kw)

    def gen(prompts: List[str]) -> List[Tuple[str, int]]:
        reqs = []
        for i, p in enumerate(prompts):
            ids, _ = render_chat(tokenizer, [{"role": "user", "content": p}], add_generation_prompt=True)
            reqs.append(GenRequest(list(ids), max_new_tokens, rid=i))
        res = eng.generate(reqs, temperature=temperature, eos_ids=eos_ids)
        return [(tokenizer.decode(r.tokens, skip_special_tokens=True), len(r.tokens)) for r in res]
    return gen


def openai_backend(url: str, model: str, *, max_new_tokens: int = 256, timeout_s: float = 120.0) -> Backend:
    """POST /v1/completions of an OpenAI-compatible server (vLLM, SGLang)."""
    def gen(prompts: List[str]) -> List[Tuple[str, int]]:
        body = json.dumps({"model": model, "prompt": prompts, "max_tokens": max_new_tokens,
                           "temperature": 0.0}).encode()
        req = urllib.request.Request(url.rstrip("/") + "/v1/completions", data=body,
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=timeout_s) as r:
            data = json.loads(r.read())
        choices = sorted(data["choices"], key=lambda c: c.get("index", 0))
        per = (data.get("usage", {}).get("completion_tokens", 0) // max(1, len(choices)))
        return [(c.get("text", ""), per) for c in choices]
    return gen
