"""Paged-KV decode kernels and the rollout engine on the GPU."""
import math

import pytest
import torch

from kore_b200.engine.rollout import GenRequest, RolloutEngine, paged_attention_reference
from kore_b200.engine.qwen3_engine import Batch, Qwen3Engine
from kore_b200.engine.smoke import smoke_config
from kore_b200.models import Qwen3Weights
from kore_b200.ops import native

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("qlens,lens,nsplit", [([1, 1, 1], [5, 300, 4099], 1), ([1, 1], [2100, 5000], 4),
                                               ([7, 1, 64], [100, 50, 64], 1)])
def test_paged_attention_vs_reference(qlens, lens, nsplit):
    torch.manual_seed(0)
    hq, hkv, D, ps = 10, 2, 128, 64
    npages = sum((L + ps - 1) // ps for L in lens) + 3
    kc = torch.randn(npages * ps, hkv, D, device="cuda").bfloat16()
    vc = torch.randn(npages * ps, hkv, D, device="cuda").bfloat16()
    perm = torch.randperm(npages).tolist()
    maxp = max((L + ps - 1) // ps for L in lens)
    bt = torch.zeros(len(lens), maxp, dtype=torch.int32)
    k = 0
    for i, L in enumerate(lens):
        n = (L + ps - 1) // ps
        bt[i, :n] = torch.tensor(perm[k:k + n], dtype=torch.int32)
        k += n
    bt = bt.cuda()
    qs = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    T = sum(qlens)
    q = torch.randn(T, hq, D, device="cuda").bfloat16()
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    po = torch.empty(nsplit * T * hq * D, device="cuda")
    pm = torch.empty(nsplit * T * hq * 2, device="cuda")
    native().paged_attention(q, kc, vc, bt, lens_t, qs, max(qlens), ps, 1 / math.sqrt(D), nsplit, out,
                             po if nsplit > 1 else None, pm if nsplit > 1 else None)
    want = paged_attention_reference(q, kc, vc, bt, lens_t, qs, ps, 1 / math.sqrt(D))
    assert _rel(out, want) < 1e-2


@pytest.mark.parametrize("hq,hkv", [(40, 8), (8, 8), (32, 4), (16, 8)])
@pytest.mark.parametrize("nsplit", [1, 3])
def test_paged_decode_groups(hq, hkv, nsplit):
    """Decode path (one query per sequence) for every GQA group size it
    specialises, including keys that end mid-chunk and empty splits."""
    torch.manual_seed(3)
    D, ps = 128, 64
    lens = [1, 31, 33, 64, 1000, 2049]
    npages = sum((L + ps - 1) // ps for L in lens) + 2
    kc = torch.randn(npages * ps, hkv, D, device="cuda").bfloat16()
    vc = torch.randn(npages * ps, hkv, D, device="cuda").bfloat16()
    perm = torch.randperm(npages).tolist()
    maxp = max((L + ps - 1) // ps for L in lens)
    bt = torch.zeros(len(lens), maxp, dtype=torch.int32)
    k = 0
    for i, L in enumerate(lens):
        n = (L + ps - 1) // ps
        bt[i, :n] = torch.tensor(perm[k:k + n], dtype=torch.int32)
        k += n
    bt = bt.cuda()
    T = len(lens)
    qs = torch.arange(T + 1, dtype=torch.int32, device="cuda")
    q = torch.randn(T, hq, D, device="cuda").bfloat16()
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    po = torch.empty(nsplit * T * hq * D, device="cuda")
    pm = torch.empty(nsplit * T * hq * 2, device="cuda")
    native().paged_attention(q, kc, vc, bt, lens_t, qs, 1, ps, 1 / math.sqrt(D), nsplit, out,
                             po if nsplit > 1 else None, pm if nsplit > 1 else None)
    want = paged_attention_reference(q, kc, vc, bt, lens_t, qs, ps, 1 / math.sqrt(D))
    assert _rel(out, want) < 1e-2


def test_sampler_device_step_matches_host_step():
    torch.manual_seed(4)
    logits = (3 * torch.randn(4, 5000, device="cuda")).bfloat16()
    t1, l1 = torch.empty(4, dtype=torch.long, device="cuda"), torch.empty(4, device="cuda")
    t2, l2 = torch.empty_like(t1), torch.empty_like(l1)
    native().sample_tokens(logits, 1.0, 0.9, 11, 7, t1, l1)
    native().sample_tokens(logits, 1.0, 0.9, 11, 0, t2, l2, torch.tensor([7], dtype=torch.int32, device="cuda"))
    assert torch.equal(t1, t2) and torch.equal(l1, l2)


def test_sampler_greedy_topp_and_logprob():
    torch.manual_seed(1)
    V = 151936
    logits = (4 * torch.randn(8, V, device="cuda")).bfloat16()
    tok = torch.empty(8, dtype=torch.long, device="cuda")
    lp = torch.empty(8, device="cuda")
    native().sample_tokens(logits, 0.0, 1.0, 0, 0, tok, lp)
    assert torch.equal(tok, logits.float().argmax(-1))
    native().sample_tokens(logits, 1.0, 1.0, 3, 1, tok, lp)
    want = torch.log_softmax(logits.float(), -1).gather(-1, tok[:, None])[:, 0]
    assert torch.allclose(lp, want, atol=1e-3)
    # tiny nucleus -> only the top token can be sampled
    native().sample_tokens(logits, 1.0, 1e-6, 5, 2, tok, lp)
    assert torch.equal(tok, logits.float().argmax(-1))
    # empirical distribution over a small vocab tracks softmax
    small = torch.tensor([[0.0, 1.0, 2.0, 3.0] * 2], device="cuda").bfloat16().repeat(4096, 1)
    t2 = torch.empty(4096, dtype=torch.long, device="cuda")
    l2 = torch.empty(4096, device="cuda")
    native().sample_tokens(small, 1.0, 1.0, 11, 3, t2, l2)
    freq = torch.bincount(t2 % 4, minlength=4).float() / 4096
    p = torch.softmax(torch.tensor([0.0, 1.0, 2.0, 3.0]), 0).cuda()
    assert (freq - p).abs().max() < 0.03


def test_rollout_greedy_matches_engine_logprobs():
    cfg = smoke_config()
    w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    eng = RolloutEngine(w, max_batch=8, page_size=64, num_pages=256, max_seq_len=2048)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (130, 77, 64)]
    outs = eng.generate([GenRequest(p, 40, rid=i, share_key="x" if i else None)
                         for i, p in enumerate(prompts)], temperature=1.0, seed=3)
    tr = Qwen3Engine(w, allocate_grads=False)
    for p, o in zip(prompts, outs):
        m = torch.zeros(len(p) + len(o.tokens), dtype=torch.bool)
        m[len(p):] = True
        b = Batch.from_sequences([torch.tensor(p + o.tokens)], [m], device="cuda")
        lp, _ = tr.token_logprobs(b)
        got = lp[b.targets >= 0].cpu()
        assert (got - torch.tensor(o.logps)).abs().mean() < 0.05
    assert len(eng.cache.free) == eng.cache.num_pages
