"""Model definitions: Qwen3 dense and Qwen3-MoE in flat per-unit buffers,
HF safetensors IO, and a plain-autograd reference forward (the oracle)."""
from .config import PRESETS, Qwen3Config, qwen3_14b, qwen3_coder_30b_a3b, qwen3_tiny
from .qwen3 import Qwen3Weights

__all__ = ["PRESETS", "Qwen3Config", "Qwen3Weights", "qwen3_14b", "qwen3_coder_30b_a3b",
           "qwen3_tiny"]
