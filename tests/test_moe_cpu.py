"""Qwen3-MoE layers in the explicit engine equal plain autograd (fp32, CPU)."""
import torch

from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
from kore_b200.models import Qwen3Config, Qwen3Weights
from kore_b200.models.reference_forward import forward_logprobs, leaf_buffers
from kore_b200.ops import moe


def tiny_moe(D=64):
    return Qwen3Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                       num_attention_heads=2, num_key_value_heads=1, head_dim=D, model_type="qwen3_moe",
                       num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                       max_position_embeddings=512, torch_dtype="float32")


def test_moe_keys_and_param_count():
    cfg = tiny_moe()
    w = Qwen3Weights(cfg, dtype=torch.float32)
    sd = w.hf_state_dict()
    assert "model.layers.0.mlp.gate.weight" in sd and "model.layers.1.mlp.experts.7.down_proj.weight" in sd
    assert sum(t.numel() for t in sd.values()) == cfg.num_params()


def test_permutation_roundtrip():
    idx = torch.tensor([[3, 1], [1, 0], [3, 2]], dtype=torch.int32)
    src, pos, offs = moe.permutation(idx, 4)
    assert offs == [0, 1, 3, 4, 6]
    assert src.tolist() == [1, 0, 1, 2, 0, 2]
    for t in range(3):
        for j in range(2):
            assert int(src[pos[t, j]]) == t
    s2, p2, o2 = moe.permutation(idx, 4, expert_range=(2, 4))
    assert o2 == [0, 1, 3] and (p2 >= 0).sum() == 3


def test_moe_engine_grads_match_autograd():
    cfg = tiny_moe()
    w = Qwen3Weights(cfg, dtype=torch.float32, seed=3)
    g = torch.Generator().manual_seed(0)
    b = Batch.from_sequences([torch.randint(0, 256, (n,), generator=g) for n in (23, 17)])
    eng = Qwen3Engine(w)
    coef = eng.sft_coef(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=coef)
    bufs = leaf_buffers(w)
    lp, _ = forward_logprobs(w, bufs, b)
    (lp * coef).sum().backward()
    for u, (gr, r) in enumerate(zip(eng.grads, bufs)):
        rel = ((gr - r.grad).norm() / (r.grad.norm() + 1e-12)).item()
        assert rel < 1e-4, (u, rel)
