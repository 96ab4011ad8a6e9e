"""Tokenizers and the Qwen ChatML template.

``load_tokenizer(model_id)`` returns the HF tokenizer when it is available
locally (no network is ever used) and otherwise a byte-level tokenizer with
the same chat special tokens, so every trainer and test runs offline.

``render_chat`` renders messages in Qwen's ChatML format and returns the ids
plus an assistant mask (1 on tokens the assistant produced), which is how
completion-only losses are built without patching the template
(the reference injects ``{% generation %}`` markers into the Jinja template
instead, kore/policy/sft.py:44-152).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>",
            "<tool_call>", "</tool_call>", "<|high_reward|>", "<|low_reward|>"]


class ByteTokenizer:
    """UTF-8 bytes (ids 0..255) + ChatML special tokens (256..)."""

    def __init__(self, vocab_size: int = 512):
        self.special = {t: 256 + i for i, t in enumerate(SPECIALS)}
        self.inv_special = {v: k for k, v in self.special.items()}
        self.vocab_size = max(vocab_size, 256 + len(SPECIALS))
        self.eos_token_id = self.special["<|im_end|>"]
        self.pad_token_id = self.special["<|endoftext|>"]
        self.name_or_path = "byte-level"

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        out: List[int] = []
        i = 0
        while i < len(text):
            hit = None
            if text[i] == "<":
                for tok, tid in self.special.items():
                    if text.startswith(tok, i):
                        hit = (tok, tid)
                        break
            if hit:
                out.append(hit[1])
                i += len(hit[0])
            else:
                j = text.find("<", i + 1)
                j = len(text) if j < 0 else j
                out.extend(text[i:j].encode("utf-8"))
                i = j
        return out

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = False) -> str:
        buf = bytearray()
        parts = []
        for t in ids:
            t = int(t)
            if t < 256:
                buf.append(t)
            else:
                if buf:
                    parts.append(buf.decode("utf-8", errors="replace"))
                    buf = bytearray()
                if not skip_special_tokens and t in self.inv_special:
                    parts.append(self.inv_special[t])
        if buf:
            parts.append(buf.decode("utf-8", errors="replace"))
        return "".join(parts)

    def __call__(self, text, **kw):
        return {"input_ids": self.encode(text)}


def load_tokenizer(model_id: Optional[str], vocab_size: int = 512):
    if model_id:
        try:
            from transformers import AutoTokenizer
            return AutoTokenizer.from_pretrained(model_id, local_files_only=True)
        except Exception:  # noqa: BLE001 - offline / not cached: byte-level fallback
            pass
    return ByteTokenizer(vocab_size)


def _enc(tok, text: str) -> List[int]:
    if isinstance(tok, ByteTokenizer):
        return tok.encode(text)
    return list(tok.encode(text, add_special_tokens=False))


def render_chat(tok, messages: List[Dict[str, str]], add_generation_prompt: bool = False,
                enable_thinking: bool = False) -> Tuple[List[int], List[int]]:
    """ChatML ids and an assistant mask (1 on assistant content + its end token)."""
    ids: List[int] = []
    mask: List[int] = []
    for m in messages:
        head = _enc(tok, f"<|im_start|>{m['role']}\n")
        body = _enc(tok, m.get("content", "") or "")
        tail = _enc(tok, "<|im_end|>")
        nl = _enc(tok, "\n")
        is_asst = m["role"] == "assistant"
        ids += head + body + tail + nl
        mask += [0] * len(head) + [1 if is_asst else 0] * (len(body) + len(tail)) + [0] * len(nl)
    if add_generation_prompt:
        g = _enc(tok, "<|im_start|>assistant\n")
        if not enable_thinking:
            g += _enc(tok, "<think>\n\n</think>\n\n")
        ids += g
        mask += [0] * len(g)
    return ids, mask


def eos_ids(tok) -> List[int]:
    out = []
    for name in ("<|im_end|>", "<|endoftext|>"):
        try:
            if isinstance(tok, ByteTokenizer):
                out.append(tok.special[name])
            else:
                out.append(tok.convert_tokens_to_ids(name))
        except Exception:  # noqa: BLE001
            pass
    return [e for e in out if e is not None and e >= 0]
