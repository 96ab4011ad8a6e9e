"""The explicit engine's forward/backward equals plain autograd (fp32, CPU)."""
import torch

from kore_b200.engine.optimizer import AdamW
from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
from kore_b200.models import Qwen3Weights, qwen3_tiny
from kore_b200.models.reference_forward import forward_logprobs, leaf_buffers


def _setup(seed=0):
    cfg = qwen3_tiny(vocab=512)
    w = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=seed)
    g = torch.Generator().manual_seed(seed)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (37, 21)]
    masks = [torch.ones(37, dtype=torch.bool), torch.arange(21) >= 10]
    return cfg, w, Batch.from_sequences(seqs, masks)


def test_batch_packing_targets():
    s = [torch.tensor([5, 6, 7]), torch.tensor([8, 9])]
    b = Batch.from_sequences(s)
    assert b.ids.tolist() == [5, 6, 7, 8, 9]
    assert b.targets.tolist() == [6, 7, -1, 9, -1]
    assert b.pos.tolist() == [0, 1, 2, 0, 1]
    assert b.cu_seqlens.tolist() == [0, 3, 5]


def test_engine_logprobs_match_reference():
    cfg, w, b = _setup()
    eng = Qwen3Engine(w)
    lp, ent = eng.token_logprobs(b, want_entropy=True)
    bufs = leaf_buffers(w)
    lp_ref, ent_ref = forward_logprobs(w, bufs, b)
    assert torch.allclose(lp, lp_ref.detach(), atol=1e-4)


def test_engine_grads_match_autograd():
    cfg, w, b = _setup(1)
    eng = Qwen3Engine(w)
    coef = eng.sft_coef(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=coef)
    bufs = leaf_buffers(w)
    lp_ref, _ = forward_logprobs(w, bufs, b)
    (lp_ref * coef).sum().backward()
    for u, (g, r) in enumerate(zip(eng.grads, bufs)):
        rel = ((g - r.grad).norm() / (r.grad.norm() + 1e-12)).item()
        assert rel < 1e-4, (u, rel)


def test_grad_accumulation_and_coef_fn():
    cfg, w, b = _setup(2)
    eng = Qwen3Engine(w)
    coef = eng.sft_coef(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=coef)
    eng.forward_backward(b, coef_fn=lambda lp: (coef, None))
    g2 = [g.clone() for g in eng.grads]
    eng.zero_grad()
    eng.forward_backward(b, coef=2 * coef)
    for a, c in zip(g2, eng.grads):
        assert torch.allclose(a, c, atol=1e-6, rtol=1e-4)


def test_sft_step_reduces_loss():
    cfg, w, b = _setup(3)
    eng = Qwen3Engine(w)
    opt = AdamW(w, eng, lr=3e-3)
    valid = b.targets >= 0
    before = -eng.token_logprobs(b)[0][valid].mean().item()
    for _ in range(3):
        eng.zero_grad()
        eng.forward_backward(b, coef=eng.sft_coef(b))
        opt.step()
    after = -eng.token_logprobs(b)[0][valid].mean().item()
    assert after < before - 0.05


def test_microbatch_grads_equal_global_token_mean():
    """Two micro-batches with coefficients -1/N_total accumulate exactly the
    gradient of one global token-mean backward over both."""
    import torch
    from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
    from kore_b200.models import Qwen3Weights, qwen3_tiny
    cfg = qwen3_tiny(vocab=256)
    w = Qwen3Weights(cfg, dtype=torch.float32, seed=1)
    g = torch.Generator().manual_seed(3)
    seqs = [torch.randint(0, 256, (n,), generator=g) for n in (20, 33, 7)]
    eng = Qwen3Engine(w)
    full = Batch.from_sequences(seqs)
    ntok = float((full.targets >= 0).sum())
    eng.zero_grad()
    eng.forward_backward(full, coef=torch.where(full.targets >= 0, -1.0 / ntok, 0.0))
    ref = [x.clone() for x in eng.grads]
    eng.zero_grad()
    for part in (seqs[:1], seqs[1:]):
        b = Batch.from_sequences(part)
        eng.forward_backward(b, coef=torch.where(b.targets >= 0, -1.0 / ntok, 0.0))
    for a, b in zip(ref, eng.grads):
        assert torch.allclose(a, b, atol=1e-6, rtol=1e-4)


def test_corrupt_checkpoint_is_skipped(tmp_path):
    import json
    import torch
    from kore_b200.models import Qwen3Weights, qwen3_tiny
    from kore_b200.models.hf_io import save_pretrained
    from kore_b200.policy.configs import latest_checkpoint
    w = Qwen3Weights(qwen3_tiny(vocab=256), dtype=torch.float32, seed=1)
    for step in (1, 2):
        save_pretrained(w, str(tmp_path / f"checkpoint-{step}"), trainer_state={"global_step": step})
    assert latest_checkpoint(str(tmp_path)).endswith("checkpoint-2")
    f = next((tmp_path / "checkpoint-2").glob("*.safetensors"))
    data = f.read_bytes()
    f.write_bytes(data[: len(data) // 2])                    # a crash mid-save
    assert latest_checkpoint(str(tmp_path)).endswith("checkpoint-1")


def test_kept_layer_contexts_match_recompute():
    """Keeping whole layer contexts (no recompute) gives the same gradients."""
    cfg, w, b = _setup(3)
    eng = Qwen3Engine(w)
    coef = eng.sft_coef(b)
    eng.zero_grad()
    eng.forward_backward(b, coef=coef)
    g_full = [g.clone() for g in eng.grads]
    for keep in (1, cfg.num_hidden_layers):
        eng.keep_layers = keep
        eng.zero_grad()
        eng.forward_backward(b, coef=coef)
        for a, c in zip(g_full, eng.grads):
            assert torch.allclose(a, c, atol=1e-6, rtol=1e-5)
    assert eng.activation_bytes_per_layer(10) > 0


def test_tp_shard_sync_in_place():
    """The TP rollout shard is refilled in place after an optimizer step and
    equals a freshly sliced shard (no new tensors)."""
    from kore_b200.parallel.tp import TPShard
    cfg = qwen3_tiny(vocab=512)
    w = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=0)
    W = 2
    for r in range(W):
        sh = TPShard(w, r, W)
        ptrs = [t.data_ptr() for L in sh.layers for t in L.values()]
        for u in range(w.num_units):
            w.bufs[u].add_(torch.randn_like(w.bufs[u]) * 0.1)
        sh.sync_from(w)
        fresh = TPShard(w, r, W)
        assert ptrs == [t.data_ptr() for L in sh.layers for t in L.values()]
        for a, b in zip(sh.layers, fresh.layers):
            for k in a:
                assert torch.equal(a[k], b[k]), k


def test_token_logprobs_many_layer_major_matches():
    """Layer-major scoring of several batches (one pass of the weights, here
    streamed through a two-slot ring) equals per-batch scoring."""
    from kore_b200.engine.frozen_stream import FrozenLayerStream
    cfg, w, b1 = _setup(3)
    _, _, b2 = _setup(4)
    eng = Qwen3Engine(w, allocate_grads=False)
    want = [eng.token_logprobs(b)[0] for b in (b1, b2)]
    ref = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, allocate=False)
    ref.bufs = [w.bufs[u].clone() if u in (0, w.num_units - 1) else None for u in range(w.num_units)]
    stream = FrozenLayerStream(ref, source="host", layers_from=w)
    reng = Qwen3Engine(ref, allocate_grads=False)
    reng.param_hook = stream
    got = [lp for lp, _ in reng.token_logprobs_many([b1, b2])]
    for a, b in zip(got, want):
        assert torch.allclose(a, b, atol=1e-5)
