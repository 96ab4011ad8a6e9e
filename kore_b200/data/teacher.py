"""Teacher models for the data factory.

* ``StubTeacher``: deterministic callable (tests, dry runs).
* ``HTTPTeacher``: any OpenAI-compatible chat endpoint (a vLLM server, a
  hosted gateway); ``ClaudeTeacher`` is the same client pointed at an
  Anthropic-compatible gateway URL / key from the environment.
* ``LocalTeacher``: a local checkpoint served by this framework's own
  rollout engine on the GPU (no external dependency).
* ``ResilientTeacher``: retries with exponential backoff and jitter, and
  trips after too many consecutive failures so a datagen run degrades
  instead of hanging.
Reference parity: kore/data/teacher.py:102-430 (Stub / vLLM / HF / Claude /
Resilient teachers and make_teacher).
"""
from __future__ import annotations

import json
import os
import random
import time
import urllib.request
from typing import Callable, List, Optional, Protocol


class TeacherClient(Protocol):
    def generate(self, messages: List[dict]) -> str: ...


def retry_call(fn: Callable, *, what: str, attempts: int = 5, base_s: float = 1.0, max_s: float = 30.0,
               stats: Optional[dict] = None):
    last = None
    for i in range(attempts):
        try:
            return fn()
        except Exception as e:  # noqa: BLE001 - network / server errors are retried
            last = e
            if stats is not None:
                stats["retries"] = stats.get("retries", 0) + 1
            if i + 1 < attempts:
                time.sleep(min(max_s, base_s * (2 ** i)) * (0.5 + random.random()))
    raise RuntimeError(f"{what} failed after {attempts} attempts: {last!r}")


class StubTeacher:
    def __init__(self, fn: Optional[Callable[[List[dict]], str]] = None):
        self.fn = fn or (lambda m: "ANALYSIS: stub\nPROPOSED_CHANGE: none\nFULL_KERNEL:\n```python\npass\n```")
        self.calls = 0

    def generate(self, messages: List[dict]) -> str:
        self.calls += 1
        return self.fn(messages)


class HTTPTeacher:
    """OpenAI-compatible /chat/completions client (urllib, no extra deps)."""

    def __init__(self, model: str, base_url: str = "http://localhost:8000/v1", api_key: Optional[str] = None,
                 temperature: float = 0.7, max_tokens: int = 8192, timeout_s: float = 600.0):
        self.model, self.base_url = model, base_url.rstrip("/")
        self.api_key = api_key or os.environ.get("OPENAI_API_KEY", "EMPTY")
        self.temperature, self.max_tokens, self.timeout = temperature, max_tokens, timeout_s
        self.stats: dict = {}

    def generate(self, messages: List[dict]) -> str:
        body = json.dumps({"model": self.model, "messages": messages, "temperature": self.temperature,
                           "max_tokens": self.max_tokens}).encode()

        def call():
            req = urllib.request.Request(f"{self.base_url}/chat/completions", data=body,
                                         headers={"Content-Type": "application/json",
                                                  "Authorization": f"Bearer {self.api_key}"})
            with urllib.request.urlopen(req, timeout=self.timeout) as r:
                d = json.loads(r.read())
            return d["choices"][0]["message"]["content"]

        t0 = time.time()
        out = retry_call(call, what="teacher call", stats=self.stats)
        self.stats["latency_s"] = time.time() - t0
        return out


class ClaudeTeacher(HTTPTeacher):
    def __init__(self, model: str = "claude", **kw):
        kw.setdefault("base_url", os.environ.get("KORE_CLAUDE_BASE_URL", "http://localhost:8080/v1"))
        kw.setdefault("api_key", os.environ.get("KORE_CLAUDE_API_KEY", ""))
        super().__init__(model, **kw)


class LocalTeacher:
    """Generation from a local checkpoint through the rollout engine."""

    def __init__(self, model_path: str, temperature: float = 0.7, max_new_tokens: int = 4096):
        import torch
        from ..data.tokenizer import eos_ids, load_tokenizer
        from ..engine.rollout import RolloutEngine
        from ..models.hf_io import from_pretrained
        self.tok = load_tokenizer(model_path)
        self.w = from_pretrained(model_path, device="cuda", dtype=torch.bfloat16)
        self.eng = RolloutEngine(self.w, max_batch=64)
        self.eos = eos_ids(self.tok)
        self.temperature, self.max_new = temperature, max_new_tokens

    def generate(self, messages: List[dict]) -> str:
        from ..data.tokenizer import render_chat
        from ..engine.rollout import GenRequest
        ids, _ = render_chat(self.tok, messages, add_generation_prompt=True)
        out = self.eng.generate([GenRequest(ids, self.max_new)], temperature=self.temperature, eos_ids=self.eos)[0]
        return self.tok.decode(out.tokens, skip_special_tokens=True)


class ResilientTeacher:
    def __init__(self, inner, max_consecutive_failures: int = 15):
        self.inner = inner
        self.max_fail = max_consecutive_failures
        self.fails = 0

    def __getattr__(self, name):
        return getattr(self.inner, name)

    def generate(self, messages, **kw) -> str:
        if self.fails >= self.max_fail:
            raise RuntimeError(f"teacher circuit open after {self.fails} consecutive failures")
        try:
            out = retry_call(lambda: self.inner.generate(messages, **kw), what="teacher", attempts=3)
            self.fails = 0
            return out
        except Exception:
            self.fails += 1
            raise


def make_teacher(kind: str = "stub", *, resilient: bool = False, **kw) -> TeacherClient:
    t = {"stub": StubTeacher, "vllm": HTTPTeacher, "http": HTTPTeacher, "claude": ClaudeTeacher,
         "local": LocalTeacher, "hf": LocalTeacher}[kind](**kw)
    return ResilientTeacher(t) if resilient else t
