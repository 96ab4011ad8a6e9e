"""GRPO step on the GPU (native kernels) with the synthetic reward env."""
import pytest
import torch

from kore_b200.engine.smoke import smoke_config
from kore_b200.env.base import SyntheticRewardEnv
from kore_b200.models import Qwen3Weights
from kore_b200.policy.configs import GRPOConfig
from kore_b200.policy.grpo import GRPOTrainer

pytestmark = pytest.mark.gpu


def test_grpo_step_gpu():
    cfg = smoke_config()
    w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    gc = GRPOConfig(num_trajectories=8, num_turns=3, tasks_per_step=2, max_response_length=64,
                    max_prompt_length=2048, learning_rate=1e-4, temperature=1.0, ref_anchor_coef=1e-2,
                    dynamic_sampling=False, starpo_s=False, total_steps=2, overlong_mask=False)
    env = SyntheticRewardEnv(seed=0, prompt_len=256, feedback_len=16, vocab_size=cfg.vocab_size)
    tr = GRPOTrainer(gc, weights=w, env=env, rollout_kwargs=dict(num_pages=512, page_size=64,
                                                                 max_seq_len=2048))
    before = [b.clone() for b in w.bufs]
    st = tr.train_step(["a", "b"])
    assert st["samples"] == 2 * 8 * 3 and st["gen_tokens"] == 2 * 8 * 3 * 64
    assert any(not torch.equal(a, b) for a, b in zip(before, w.bufs))
    st2 = tr.train_step(["c", "d"])
    assert st2["kl"] > 0 and torch.isfinite(torch.tensor(st2["loss"]))
