"""Model configurations (HF ``config.json`` field names) for the Qwen3 dense
and Qwen3-MoE decoders.

The reference loads these architectures through ``AutoModelForCausalLM``
(kore/policy/grpo.py:2017-2018, kore/policy/sft.py:288-293) and detects the
decoder layer class by name (kore/policy/configs.py:550-567). Here the model
code is our own; the config keeps HF's field names so ``config.json`` files
round-trip.
"""
from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field, fields
from typing import Optional


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 5120
    intermediate_size: int = 17408
    num_hidden_layers: int = 40
    num_attention_heads: int = 40
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False
    torch_dtype: str = "bfloat16"
    model_type: str = "qwen3"
    architectures: list = field(default_factory=lambda: ["Qwen3ForCausalLM"])
    # MoE fields (used when model_type == "qwen3_moe")
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: list = field(default_factory=list)
    router_aux_loss_coef: float = 0.001
    bos_token_id: Optional[int] = 151643
    eos_token_id: Optional[int] = 151645

    @property
    def is_moe(self) -> bool:
        return self.model_type == "qwen3_moe" and self.num_experts > 0

    def layer_is_moe(self, i: int) -> bool:
        if not self.is_moe or i in (self.mlp_only_layers or []):
            return False
        return (i + 1) % max(1, self.decoder_sparse_step) == 0

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def num_params(self) -> int:
        H, V = self.hidden_size, self.vocab_size
        attn = H * (self.q_dim + 2 * self.kv_dim) + self.q_dim * H + 2 * self.head_dim
        total = V * H * (1 if self.tie_word_embeddings else 2) + H
        for i in range(self.num_hidden_layers):
            if self.layer_is_moe(i):
                mlp = self.num_experts * 3 * H * self.moe_intermediate_size + self.num_experts * H
            else:
                mlp = 3 * H * self.intermediate_size
            total += attn + mlp + 2 * H
        return total

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "Qwen3Config":
        names = {f.name for f in fields(cls)}
        kw = {k: v for k, v in d.items() if k in names}
        if "head_dim" not in d and "hidden_size" in d and "num_attention_heads" in d:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        return cls(**kw)

    @classmethod
    def from_pretrained(cls, path: str) -> "Qwen3Config":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_dict(json.load(f))

    def save(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(self.to_dict(), f, indent=2)


def qwen3_14b() -> Qwen3Config:
    """Qwen3-14B architecture (40 layers, hidden 5120, 40 Q / 8 KV heads)."""
    return Qwen3Config()


def qwen3_tiny(vocab: int = 32000) -> Qwen3Config:
    """The tiny CPU policy of the gloo GRPO smoke: 2 layers, hidden 256,
    4 Q / 2 KV heads, FFN 704, vocab 32000."""
    return Qwen3Config(vocab_size=vocab, hidden_size=256, intermediate_size=704,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=64, max_position_embeddings=4096, torch_dtype="float32")


def qwen3_coder_30b_a3b() -> Qwen3Config:
    """Qwen3-Coder-30B-A3B architecture (48 layers, hidden 2048, 32 Q / 4 KV,
    128 experts top-8, expert FFN 768)."""
    return Qwen3Config(vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                       num_hidden_layers=48, num_attention_heads=32, num_key_value_heads=4,
                       head_dim=128, model_type="qwen3_moe",
                       architectures=["Qwen3MoeForCausalLM"], num_experts=128,
                       num_experts_per_tok=8, moe_intermediate_size=768, max_position_embeddings=262144)


PRESETS = {
    "qwen3-14b": qwen3_14b,
    "qwen3-tiny": qwen3_tiny,
    "qwen3-coder-30b-a3b": qwen3_coder_30b_a3b,
}
