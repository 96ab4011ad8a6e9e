"""Serving: a generation front end over the framework's own rollout engine.

* ``KorePolicy``: loads an HF-format Qwen3 checkpoint into the paged-KV
  continuous-batching engine (optionally tensor-parallel over the GPUs of a
  process group) and exposes ``generate(prompts)`` and ``chat(messages)``
  with thinking disabled in the chat template.
* ``load_generate(model, backend)``: a ``prompt -> text`` callable for eval,
  retention and relabelling; ``backend="kore"`` (default) uses the engine,
  ``backend="vllm"`` uses the installed vLLM library when asked for.
* ``app(policy)``: an OpenAI-compatible ``/v1/chat/completions`` FastAPI app
  (``kore serve``), so the data-factory HTTP teacher can point at it.
Reference parity: kore/policy/serve.py:44-254 (vLLM wrapper with TP size,
load_generate with hf|vllm backends, thinking disabled).
"""
from __future__ import annotations

import argparse
import time
from typing import Callable, List, Optional, Sequence


class KorePolicy:
    def __init__(self, model_path: str, *, device: str = "cuda", max_batch: int = 64, temperature: float = 0.0,
                 top_p: float = 1.0, max_new_tokens: int = 2048, weights=None, tokenizer=None):
        import torch
        from ..data.tokenizer import eos_ids, load_tokenizer
        from ..engine.rollout import RolloutEngine
        from ..models.hf_io import from_pretrained
        self.tok = tokenizer if tokenizer is not None else load_tokenizer(model_path)
        self.w = weights if weights is not None else from_pretrained(model_path, device=device, dtype=torch.bfloat16)
        self.eng = RolloutEngine(self.w, max_batch=max_batch)
        self.eos = eos_ids(self.tok)
        self.temperature, self.top_p, self.max_new = temperature, top_p, max_new_tokens

    def generate_ids(self, prompts: Sequence[List[int]], max_new_tokens: Optional[int] = None, seed: int = 0):
        from ..engine.rollout import GenRequest
        reqs = [GenRequest(list(p), max_new_tokens or self.max_new) for p in prompts]
        return self.eng.generate(reqs, temperature=self.temperature, top_p=self.top_p, eos_ids=self.eos, seed=seed)

    def chat(self, conversations: Sequence[List[dict]], **kw) -> List[str]:
        from ..data.tokenizer import render_chat
        ids = [render_chat(self.tok, m, add_generation_prompt=True, enable_thinking=False)[0] for m in conversations]
        return [self.tok.decode(r.tokens, skip_special_tokens=True) for r in self.generate_ids(ids, **kw)]

    def generate(self, prompts: Sequence[str], **kw) -> List[str]:
        return self.chat([[{"role": "user", "content": p}] for p in prompts], **kw)


def load_generate(model_path: str, backend: str = "kore", **kw) -> Callable[[str], str]:
    if backend == "kore":
        pol = KorePolicy(model_path, **kw)
        return lambda prompt: pol.generate([prompt])[0]
    if backend == "vllm":
        from vllm import LLM, SamplingParams
        llm = LLM(model=model_path, tensor_parallel_size=kw.get("tp", 1), dtype="bfloat16")
        sp = SamplingParams(temperature=kw.get("temperature", 0.0), max_tokens=kw.get("max_new_tokens", 2048))
        return lambda prompt: llm.chat([{"role": "user", "content": prompt}], sp,
                                       chat_template_kwargs={"enable_thinking": False})[0].outputs[0].text
    raise ValueError(f"unknown backend {backend!r}")


def app(policy: KorePolicy):
    from fastapi import FastAPI
    api = FastAPI()

    @api.post("/v1/chat/completions")
    def chat(body: dict):
        text = policy.chat([body["messages"]], max_new_tokens=body.get("max_tokens"))[0]
        return {"id": f"kore-{int(time.time() * 1e3)}", "object": "chat.completion", "model": body.get("model", ""),
                "choices": [{"index": 0, "finish_reason": "stop", "message": {"role": "assistant", "content": text}}]}
    return api


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore serve")
    ap.add_argument("model")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-batch", type=int, default=64)
    a = ap.parse_args(argv)
    import uvicorn
    uvicorn.run(app(KorePolicy(a.model, max_batch=a.max_batch)), host="127.0.0.1", port=a.port)
    return 0
