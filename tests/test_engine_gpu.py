"""The explicit engine on the GPU (native kernels, bf16) against the fp32
autograd reference forward."""
import pytest
import torch

from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
from kore_b200.engine.smoke import run_smoke, smoke_config
from kore_b200.models import Qwen3Weights
from kore_b200.models.reference_forward import forward_logprobs, leaf_buffers

pytestmark = pytest.mark.gpu


def _batch(cfg, seed, lens=(200, 120)):
    g = torch.Generator().manual_seed(seed)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in lens]
    return Batch.from_sequences(seqs, device="cuda")


def test_engine_gpu_grads_vs_fp32_reference():
    cfg = smoke_config()
    w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    b = _batch(cfg, 0)
    eng = Qwen3Engine(w, grad_dtype=torch.float32)
    lp, _ = eng.token_logprobs(b)
    bufs = leaf_buffers(w)
    lp_ref, _ = forward_logprobs(w, bufs, b)
    assert (lp - lp_ref.detach()).abs().max().item() < 0.05
    coef = eng.sft_coef(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=coef)
    (lp_ref * coef).sum().backward()
    for u, (gr, r) in enumerate(zip(eng.grads, bufs)):
        rel = ((gr.float() - r.grad).norm() / (r.grad.norm() + 1e-12)).item()
        assert rel < 3e-2, (u, rel)


def test_smoke():
    out = run_smoke("cuda:0")
    assert out["loss_after"] < out["loss_before"]
