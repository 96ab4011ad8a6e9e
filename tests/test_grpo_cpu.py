"""GRPO trainer, rollout engine and HF checkpoints on a tiny fp32 model (CPU)."""
import pytest
import json
import os

import torch

from kore_b200.engine.qwen3_engine import Batch
from kore_b200.engine.rollout import (GenRequest, RolloutEngine, paged_attention_reference)
from kore_b200.env.base import SyntheticRewardEnv
from kore_b200.models import Qwen3Weights, qwen3_tiny
from kore_b200.models.hf_io import from_pretrained, save_pretrained
from kore_b200.models.reference_forward import forward_logprobs, leaf_buffers
from kore_b200.ops import reference as ref
from kore_b200.policy.configs import GRPOConfig
from kore_b200.policy.grpo import GRPOTrainer


def _tiny(vocab=512, seed=0):
    cfg = qwen3_tiny(vocab=vocab)
    return cfg, Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=seed)


def test_rollout_greedy_matches_full_forward():
    cfg, w = _tiny()
    eng = RolloutEngine(w, max_batch=4, page_size=16, num_pages=64, max_seq_len=512)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 33)]
    outs = eng.generate([GenRequest(p, 6, rid=i) for i, p in enumerate(prompts)], temperature=0.0)
    bufs = leaf_buffers(w)
    for p, o in zip(prompts, outs):
        seq = list(p)
        for t in o.tokens:  # greedy: each token is the argmax of the full recompute
            b = Batch.from_sequences([torch.tensor(seq + [0])])
            x = _logits_last(w, bufs, b)
            assert int(x.argmax()) == t
            seq.append(t)
    assert all(len(o.tokens) == 6 for o in outs)
    assert len(eng.cache.free) == eng.cache.num_pages  # every page returned


def _logits_last(w, bufs, b):
    import kore_b200.models.reference_forward as rf
    cfg = w.cfg
    with torch.no_grad():
        lp_all = []
        # full-vocab logits at the last real position via the oracle forward
        V = [lay.views(t) for lay, t in zip(w.layouts, bufs)]
        x = V[0]["embed"][b.ids]
        T = x.shape[0]
        hq, hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        cos, sin = ref.rope_tables(cfg.max_position_embeddings, D, cfg.rope_theta)
        for u in range(1, len(bufs) - 1):
            W = V[u]
            hn = ref.rmsnorm(x, W["ln1"], cfg.rms_norm_eps)
            qkv = hn @ W["qkv"].t()
            qk = ref.qk_norm_rope(qkv, W["q_norm"], W["k_norm"], b.pos, cos, sin, hq, hkv, cfg.rms_norm_eps)
            o = ref.causal_attention(qk[:, :hq * D].reshape(T, hq, D), qk[:, hq * D:].reshape(T, hkv, D),
                                     qkv[:, (hq + hkv) * D:].reshape(T, hkv, D), cu_seqlens=b.cu_seqlens)
            x = x + o.reshape(T, -1) @ W["o"].t()
            x = x + ref.swiglu(ref.rmsnorm(x, W["ln2"], cfg.rms_norm_eps) @ W["gate_up"].t()) @ W["down"].t()
        h = ref.rmsnorm(x, V[-1]["norm"], cfg.rms_norm_eps)
        return (h @ V[-1]["lm_head"].t())[-2]


def test_prefix_sharing_returns_pages():
    cfg, w = _tiny()
    eng = RolloutEngine(w, max_batch=8, page_size=8, num_pages=128, max_seq_len=512)
    p = list(range(1, 30))
    outs = eng.generate([GenRequest(p, 4, rid=i, share_key="t") for i in range(4)], temperature=0.0)
    assert len({tuple(o.tokens) for o in outs}) == 1   # identical greedy continuations
    assert len(eng.cache.free) == eng.cache.num_pages


def test_grpo_step_cpu_tiny():
    cfg, w = _tiny()
    gc = GRPOConfig(num_trajectories=4, num_turns=2, tasks_per_step=2, max_response_length=8,
                    max_prompt_length=256, learning_rate=1e-3, temperature=1.0, ref_anchor_coef=1e-2,
                    dynamic_sampling=False, starpo_s=False, bf16=False, total_steps=2,
                    overlong_mask=False)
    env = SyntheticRewardEnv(seed=0, prompt_len=16, feedback_len=4, vocab_size=cfg.vocab_size)
    tr = GRPOTrainer(gc, weights=w, env=env, rollout_kwargs=dict(num_pages=256, page_size=16,
                                                                 max_seq_len=512))
    before = [b.clone() for b in w.bufs]
    st = tr.train_step(["a", "b"])
    assert st["samples"] == 2 * 4 * 2 and st["groups"] == 2
    assert any(not torch.equal(a, b) for a, b in zip(before, w.bufs))
    assert st["kl"] >= 0


def test_hf_checkpoint_roundtrip(tmp_path):
    cfg, w = _tiny()
    save_pretrained(w, str(tmp_path / "ck"))
    with open(tmp_path / "ck" / "config.json") as f:
        assert json.load(f)["model_type"] == "qwen3"
    w2 = from_pretrained(str(tmp_path / "ck"), dtype=torch.float32)
    for a, b in zip(w.hf_state_dict().values(), w2.hf_state_dict().values()):
        assert torch.equal(a, b)
    keys = set(w.hf_state_dict())
    assert "model.layers.0.self_attn.q_proj.weight" in keys and "lm_head.weight" in keys
    assert "model.layers.1.mlp.down_proj.weight" in keys


def test_grpo_resume_restores_optimizer_and_rng(tmp_path):
    """A GRPO run checkpoints weights, optimizer shard and RNG; a restarted run
    resumes at the saved step with the same optimizer step count."""
    from kore_b200.policy.grpo import train_grpo
    cfg, _ = _tiny()
    out = str(tmp_path / "run")
    kw = dict(num_trajectories=2, num_turns=1, tasks_per_step=1, max_response_length=4, max_prompt_length=64,
              learning_rate=1e-3, dynamic_sampling=False, starpo_s=False, bf16=False, overlong_mask=False,
              save_steps=1, output_dir=out, model_id="tiny-test")
    env = SyntheticRewardEnv(seed=0, prompt_len=8, feedback_len=2, vocab_size=cfg.vocab_size)
    r1 = train_grpo(GRPOConfig(total_steps=2, **kw), env=env, model_cfg=cfg)
    assert len(r1["history"]) == 2
    st = torch.load(f"{out}/checkpoint-2/grpo_state-rank0.pt", weights_only=False)
    assert st["opt"]["step"] == 2
    r2 = train_grpo(GRPOConfig(total_steps=3, **kw), env=env, model_cfg=cfg)
    assert len(r2["history"]) == 1                       # resumed at step 2, ran step 3 only


def test_multiturn_graph_rollout_matches_turnwise_engine():
    """The batched multi-turn rollout (decode loop over device-resident state)
    generates the same greedy transcripts as turn-by-turn engine calls."""
    from kore_b200.engine.multiturn import MultiTurnRollout
    cfg, w = _tiny()
    g = torch.Generator().manual_seed(1)
    base = [torch.randint(0, cfg.vocab_size, (18,), generator=g).tolist() for _ in range(2)]
    prompts = [list(base[0]), list(base[0]), list(base[1])]
    fb = lambda turn, i, gen: [(7 * turn + i + k) % cfg.vocab_size for k in range(3)]
    eng = RolloutEngine(w, max_batch=8, page_size=16, num_pages=128, max_seq_len=512)
    outs = MultiTurnRollout(eng, poll=3).run(prompts, num_turns=3, max_new=5, feedback=fb,
                                             share_keys=[0, 0, 1], max_feedback=3, temperature=0.0)
    assert len(eng.cache.free) == eng.cache.num_pages
    ref_eng = RolloutEngine(w, max_batch=8, page_size=16, num_pages=128, max_seq_len=512)
    ctx = [list(p) for p in prompts]
    for turn in range(3):
        res = ref_eng.generate([GenRequest(c, 5, rid=i) for i, c in enumerate(ctx)], temperature=0.0)
        for i, r in enumerate(res):
            assert outs[i].contexts[turn] == ctx[i]
            assert outs[i].gens[turn] == r.tokens, (turn, i)
            for a, b in zip(outs[i].logps[turn], r.logps):
                assert abs(a - b) < 1e-4
            ctx[i] = ctx[i] + r.tokens + fb(turn, i, r.tokens)


def test_grpo_trajectory_packing_same_gradient():
    """Training all turns of a trajectory in one packed row gives the same
    gradient as one sequence per turn sample."""
    cfg, w = _tiny()
    gc = GRPOConfig(num_trajectories=2, num_turns=2, tasks_per_step=1, max_response_length=6,
                    max_prompt_length=256, max_feedback_tokens=4, learning_rate=1e-3, temperature=1.0,
                    ref_anchor_coef=1e-2, dynamic_sampling=False, starpo_s=False, bf16=False,
                    overlong_mask=False)
    env = SyntheticRewardEnv(seed=0, prompt_len=12, feedback_len=4, vocab_size=cfg.vocab_size)
    tr = GRPOTrainer(gc, weights=w, env=env, rollout_kwargs=dict(num_pages=256, page_size=16,
                                                                 max_seq_len=512))
    assert tr._batched_ok(6)
    groups = tr.rollout_batch(["a"], [0, 1], max_new_tokens=6)
    samples = tr.samples_from_group(groups[0], 0)
    assert len(tr._rows(samples)) == 2            # two trajectories -> two packed rows
    for s in samples:
        s.adv = 0.5 if s.turn == 0 else -0.25
    tr.fill_ref_logps(samples, 4096)
    tr.trainer.opt.step = lambda *a, **k: None
    grads = {}
    for pack in (True, False):
        tr.cfg.pack_trajectories = pack
        tr.update(samples, 4096)
        grads[pack] = [g.clone() for g in tr.trainer.eng.grads]
    for a, b in zip(grads[True], grads[False]):
        assert torch.allclose(a, b, atol=1e-6, rtol=1e-4)
    assert any(g.abs().sum() > 0 for g in grads[True])


def test_grpo_streamed_reference_matches_resident():
    """The frozen KL reference streamed layer by layer scores like a resident copy."""
    cfg, w = _tiny()
    env = SyntheticRewardEnv(seed=0, prompt_len=12, feedback_len=4, vocab_size=cfg.vocab_size)
    base = dict(num_trajectories=2, num_turns=1, tasks_per_step=1, max_response_length=6, max_prompt_length=256,
                max_feedback_tokens=4, learning_rate=1e-3, temperature=1.0, ref_anchor_coef=1e-2,
                dynamic_sampling=False, starpo_s=False, bf16=False, overlong_mask=False)
    res = {}
    for place in ("resident", "host"):
        tr = GRPOTrainer(GRPOConfig(ref_placement=place, **base), weights=w.clone(), env=env,
                         rollout_kwargs=dict(num_pages=128, page_size=16, max_seq_len=512))
        assert tr.ref_placement == place
        groups = tr.rollout_batch(["a"], [0, 1], max_new_tokens=6)
        samples = tr.samples_from_group(groups[0], 0)
        tr.fill_ref_logps(samples, 4096)
        res[place] = [s.ref_logp for s in samples]
    assert res["resident"] == pytest.approx(res["host"], abs=1e-5)


def test_grpo_update_gradient_matches_autograd_objective():
    """The update's gradient equals autograd of the GRPO objective written
    out directly: per sample the token-mean log-prob lp, ratio r = e^(lp - old),
    term = -min(r A, clip(r, 1 - lo, 1 + hi) A) + c (e^(ref - lp) - (ref - lp) - 1),
    loss = sum_s n_s term_s / total tokens. Old log-probs are offset so that
    some ratios sit outside the clip band."""
    from kore_b200.policy.grpo import TrainSample
    cfg, w = _tiny()
    lo, hi, c = 0.2, 0.28, 0.05
    gc = GRPOConfig(num_trajectories=4, num_turns=1, tasks_per_step=1, max_response_length=8,
                    max_prompt_length=256, learning_rate=1e-3, clip_ratio_low=lo, clip_ratio_high=hi,
                    ref_anchor_coef=c, old_logp_source="sampler", dynamic_sampling=False, starpo_s=False,
                    bf16=False, total_steps=2, overlong_mask=False)
    env = SyntheticRewardEnv(seed=0, prompt_len=16, feedback_len=4, vocab_size=cfg.vocab_size)
    tr = GRPOTrainer(gc, weights=w, env=env, rollout_kwargs=dict(num_pages=64, page_size=16, max_seq_len=256))
    g = torch.Generator().manual_seed(3)
    adv = [1.0, 0.5, -0.8, -1.2]           # samples 1 and 2 land on the clipped branch
    offs = [0.0, 0.3, -0.3, 0.05]                   # old = lp - off: r = e^off
    samples, lps = [], []
    bufs = leaf_buffers(w)
    for i in range(4):
        L, n_ctx = 20 + 3 * i, 8 + i
        ids = torch.randint(0, cfg.vocab_size, (L,), generator=g).tolist()
        # the policy's log-probs at the sampling temperature, as the update scores them
        lp, _ = forward_logprobs(w, bufs, Batch.from_sequences([torch.tensor(ids)]), temperature=gc.temperature)
        m = lp[n_ctx - 1: L - 1].mean()
        lps.append(m)
        samples.append(TrainSample(ids, n_ctx, ret=0.0, adv=adv[i], old_logp=m.item() - offs[i],
                                   ref_logp=m.item() + 0.1))
    total = sum(s.n_gen for s in samples)
    loss = 0.0
    for s, m in zip(samples, lps):
        r = torch.exp(m - s.old_logp)
        pg = -torch.minimum(r * s.adv, r.clamp(1 - lo, 1 + hi) * s.adv)
        d = s.ref_logp - m
        loss = loss + s.n_gen * (pg + c * (torch.exp(d) - d - 1)) / total
    loss.backward()
    tr.trainer.opt.step = lambda *a, **k: None
    st = tr.update(samples, budget=4096)
    assert abs(st["loss"] - float(loss)) < 1e-5 * max(1.0, abs(float(loss)))
    for u, (gr, rb) in enumerate(zip(tr.trainer.eng.grads, bufs)):
        rel = ((gr - rb.grad).norm() / (rb.grad.norm() + 1e-12)).item()
        assert rel < 1e-4, (u, rel)
