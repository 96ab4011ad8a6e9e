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


def test_multiturn_graph_rollout_gpu():
    """CUDA-graph decode loop vs turn-by-turn engine calls (greedy, bf16):
    transcripts agree and the sampled log-probs match where they agree."""
    from kore_b200.engine.multiturn import MultiTurnRollout
    from kore_b200.engine.rollout import GenRequest, RolloutEngine
    from kore_b200.ops import check_device_error
    cfg = smoke_config()
    w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=1)
    g = torch.Generator().manual_seed(5)
    base = [torch.randint(0, cfg.vocab_size, (130,), generator=g).tolist() for _ in range(3)]
    prompts = [base[i // 4] for i in range(12)]
    fb = lambda turn, i, gen: [(31 * turn + 7 * i + k) % cfg.vocab_size for k in range(9)]
    eng = RolloutEngine(w, max_batch=16, page_size=64, num_pages=256, max_seq_len=2048)
    outs = MultiTurnRollout(eng, poll=16).run(prompts, num_turns=3, max_new=40, feedback=fb,
                                              share_keys=[i // 4 for i in range(12)], max_feedback=9,
                                              temperature=0.0)
    assert check_device_error() == 0
    # teacher forcing: the training engine scores the transcripts the graph loop produced;
    # greedy sampling reports log-probs of the untempered softmax
    from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
    scorer = Qwen3Engine(w, allocate_grads=False)
    err, n = 0.0, 0
    for o in outs:
        full = o.contexts[-1] + o.gens[-1]
        b = Batch.from_sequences([torch.tensor(full)], device="cuda")
        lp, _ = scorer.token_logprobs(b)
        lp = lp.float().cpu()
        for t in range(3):
            c0 = len(o.contexts[t])
            for j, v in enumerate(o.logps[t]):
                err = max(err, abs(v - float(lp[c0 - 1 + j])))
                n += 1
    assert n == 12 * 3 * 40 and err < 6e-2, err
    assert len(eng.cache.free) == eng.cache.num_pages
