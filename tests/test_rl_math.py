"""Pure GRPO / anti-collapse math (CPU)."""
import math

import pytest
import torch

from kore_b200.policy import rl_math as M
from kore_b200.reward.shaping import discounted_shaping_sum, shaped_turn_rewards, shaping_terms


def test_group_advantages_and_degenerate():
    a = M.group_advantages([1.0, 2.0, 3.0])
    assert abs(sum(a)) < 1e-9 and a[0] < 0 < a[2]
    assert all(abs(x) < 1e-6 for x in M.group_advantages([0.5, 0.5, 0.5]))


def test_discounted_returns():
    assert M.discounted_returns([1.0, 0.0, 1.0], 0.5) == pytest.approx([1.25, 0.5, 1.0])


def test_clip_higher_float_and_tensor():
    assert M.clip_higher_ratio(1.5, 1.0, 0.2, 0.28) == pytest.approx(1.28)
    assert M.clip_higher_ratio(0.5, -1.0, 0.2, 0.28) == pytest.approx(-0.8)
    r = torch.tensor(1.5, requires_grad=True)
    out = M.clip_higher_ratio(r, 1.0, 0.2, 0.28)
    out.backward()
    assert r.grad.item() == 0.0  # clipped region: zero gradient, graph kept


def test_kevin_credit_and_infra_drop():
    assert M.kevin_trajectory_score([0.5, 1.0, 0.2], [True, False, True]) == 0.5
    rets, idx = M.build_kevin_samples([[1.0, 2.0]], [[False, True]], gamma=0.4, traj_infra=[[True, False]])
    assert idx == [(0, 1)] and rets == pytest.approx([2.0])
    r = M.kevin_turn_returns([0.03, 1.0], [False, True], 0.4, credit_incorrect=True)
    assert r[0] == pytest.approx(0.03 + 0.4)


def test_pbs_telescopes():
    phis = [0.2, 0.5, 0.7]
    assert discounted_shaping_sum(phis, 0.4) == pytest.approx(-0.2)
    assert shaping_terms([0.1, None, 0.3], 0.5)[0] == 0.0
    assert shaped_turn_rewards([1, 1], [0.0, 0.5], 0.5, 2.0)[0] == pytest.approx(1 + 2 * 0.25)


def test_starpo_and_refill():
    groups = [[1, 1, 1], [0, 1, 0], [0, 5, 0], [2, 2.1, 2]]
    keep = M.starpo_select_high_variance(groups, keep_frac=0.5)
    assert keep == [1, 2]
    seq = iter([[1, 1], [0, 1], [2, 2], [0, 3]])
    kept, att = M.dynamic_sampling_refill(lambda i: next(seq), 2)
    assert kept == [[0, 1], [0, 3]] and att == 4


def test_avspo_floor_and_cross_rank():
    adv = M.avspo_advantages([1.0, 1.0001], tau=0.1, k=2)
    assert max(abs(a) for a in adv) < 0.01  # virtual samples bound the advantage
    per_rank = [[1.0, 2.0], [3.0], [0.0, 4.0]]
    split = M.distributed_group_advantages(per_rank)
    flat = M.avspo_advantages([1.0, 2.0, 3.0, 0.0, 4.0], 0.0)
    assert [x for c in split for x in c] == pytest.approx(flat)
    assert M.rank_slice(8, 1, 4) == [1, 5]


def test_rc_sc_gtpo():
    toks = M.sample_reward_tokens(8, 0.5, seed=0)
    assert toks.count(M.HIGH_REWARD_TOKEN) == 4
    assert M.scgrpo_weight_from_kl([]) == 1.0
    assert M.scgrpo_weight_from_kl([10.0]) == 2.0
    sh = M.gtpo_codesim_shaping(["a = b + c", "x"], ["a = b + c"], scale=0.3)
    assert sh[0] == pytest.approx(0.3) and sh[1] < 0.3


def test_kl_k3_and_overlong():
    assert M.kl_k3(0.0, 0.0) == 0.0 and M.kl_k3(-1.0, 0.0) > 0
    assert M.is_overlong(1900, 2048, 200) and not M.is_overlong(100, 2048, 200)
    assert not M.is_overlong(10 ** 6, 0, 10)


def test_dynamic_step_controller():
    c = M.DynamicStepController(min_steps=2, max_steps=100, patience=2)
    assert not c.update(0, 1.0) and not c.update(1, 1.0)
    assert c.update(2, 1.0) and "plateau" in c.stopped_reason


@pytest.mark.parametrize("has_old", [True, False])
def test_grpo_token_coefficients_match_autograd(has_old):
    torch.manual_seed(0)
    samples, lps = [], []
    for i in range(6):
        samples.append(M.GRPOSample(adv=float(torch.randn(())), n_tokens=3 + i,
                                    old_logp=(-1.0 + 0.05 * i) if has_old else None,
                                    ref_logp=-1.1, sc_weight=1.0 + 0.1 * i))
        lps.append(-1.0 + 0.07 * (i - 3))
    total = sum(s.n_tokens for s in samples)
    loss, coefs = M.grpo_token_coefficients(samples, lps, clip_lo=0.03, clip_hi=0.04, ref_coef=1e-3,
                                            total_tokens=total)
    # autograd over per-token logps whose token mean is lp
    terms = 0.0
    grads = []
    for s, lp in zip(samples, lps):
        tok = torch.full((s.n_tokens,), lp, dtype=torch.float64, requires_grad=True)
        m = tok.mean()
        if s.old_logp is not None:
            r = torch.exp(m - s.old_logp)
            pg = -M.clip_higher_ratio(r, s.adv, 0.03, 0.04)
        else:
            pg = -s.adv * m
        pg = pg * s.sc_weight
        d = s.ref_logp - m
        t = (pg + 1e-3 * (torch.exp(d) - d - 1)) * s.n_tokens / total
        t.backward()
        terms += float(t)
        grads.append(tok.grad)
    assert loss == pytest.approx(terms, rel=1e-9, abs=1e-12)
    for c, g in zip(coefs, grads):
        assert torch.allclose(g, torch.full_like(g, c), rtol=1e-9, atol=1e-12)
