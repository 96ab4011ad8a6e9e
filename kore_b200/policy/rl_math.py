"""Pure RL math of the GRPO trainer (torch-free except where noted).

Behavioural parity with the reference's GRPO / anti-collapse math; each
function cites the reference function whose behaviour it reproduces:

* group-relative advantages, discounted turn returns, Kevin credit
  (kore/policy/grpo.py:31-191)
* DAPO clip-higher surrogate, overlong masking, dynamic-sampling refill
  (kore/policy/grpo.py:52-83, :270-299)
* StarPO-S high-variance group selection (kore/policy/grpo.py:241-267)
* k3 KL anchor, value prefilter (kore/policy/grpo.py:305-328)
* cross-rank group advantages and strided rank slices
  (kore/policy/grpo.py:1484-1559)
* AVSPO / RC-GRPO / SC-GRPO / GTPO anti-collapse ladder
  (kore/policy/anticollapse.py:41-213)
* plateau early stop (kore/policy/dynamic.py:21-51)

On top of that, :func:`grpo_token_coefficients` turns the per-sample GRPO
objective into the per-token coefficients ``dL/dlogp_t`` the explicit engine
consumes (its backward never builds an autograd graph).
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

EPS = 1e-6


# ---------------------------------------------------------------- advantages
def group_advantages(rewards: Sequence[float], eps: float = EPS) -> List[float]:
    """(r - mean) / (population std + eps); an all-equal group gives ~0."""
    n = len(rewards)
    if n == 0:
        return []
    mu = sum(rewards) / n
    sd = math.sqrt(sum((r - mu) ** 2 for r in rewards) / n)
    return [(r - mu) / (sd + eps) for r in rewards]


def discounted_returns(scores: Sequence[float], gamma: float = 0.4) -> List[float]:
    """R_t = s_t + gamma * R_{t+1}, computed right to left."""
    out = [0.0] * len(scores)
    acc = 0.0
    for t in reversed(range(len(scores))):
        acc = scores[t] + gamma * acc
        out[t] = acc
    return out


def clip_higher_ratio(ratio, advantage, lo: float = 0.2, hi: float = 0.28):
    """min(r*A, clip(r, 1-lo, 1+hi)*A); works on floats and torch tensors."""
    if hasattr(ratio, "clamp"):
        import torch
        return torch.minimum(ratio * advantage, ratio.clamp(1.0 - lo, 1.0 + hi) * advantage)
    c = min(max(ratio, 1.0 - lo), 1.0 + hi)
    return min(ratio * advantage, c * advantage)


def is_overlong(n_tokens: int, max_response_length: int, buffer_len: int) -> bool:
    """True when a response ends within ``buffer_len`` tokens of the cap
    (almost surely truncated); never when the cap is unset."""
    if not max_response_length or max_response_length <= 0:
        return False
    return n_tokens >= max(1, int(max_response_length) - max(0, int(buffer_len)))


def kevin_trajectory_score(turn_rewards: Sequence[float], correct: Sequence[bool]) -> float:
    """A trajectory is worth its best correct turn (0 when none is correct)."""
    good = [r for r, c in zip(turn_rewards, correct) if c]
    return max(good) if good else 0.0


def kevin_turn_returns(turn_rewards, correct, gamma: float = 0.4, *,
                       credit_incorrect: bool = False, phis=None,
                       phi_weight: float = 0.0) -> List[float]:
    """Correctness-gated per-turn returns with optional potential shaping.

    Incorrect turns contribute 0 unless ``credit_incorrect`` keeps their
    (bounded, sub-threshold) shaped reward. With ``phis`` (exit potentials
    per turn) and ``phi_weight`` the PBS term w*(gamma*Phi(s_{t+1}) - Phi(s_t))
    is added, with the entering potential of turn t = exit potential of t-1
    (0 for the first turn)."""
    from ..reward.shaping import shaping_terms
    base = [float(r) if (c or credit_incorrect) else 0.0 for r, c in zip(turn_rewards, correct)]
    if phis is not None and phi_weight:
        enter = [0.0] + list(phis)[:-1]
        terms = shaping_terms(enter, gamma)
        base = [b + phi_weight * (terms[t] if t < len(terms) else 0.0) for t, b in enumerate(base)]
    return discounted_returns(base, gamma)


def build_kevin_samples(traj_rewards, traj_correct, gamma: float = 0.4, traj_infra=None, *,
                        credit_incorrect: bool = False, traj_phis=None,
                        phi_weight: float = 0.0) -> Tuple[List[float], List[Tuple[int, int]]]:
    """Flatten trajectories x turns into per-turn samples; turns flagged as
    infrastructure failures are dropped (they stay in the gamma chain with 0)."""
    rets: List[float] = []
    idx: List[Tuple[int, int]] = []
    for ti, (rw, cr) in enumerate(zip(traj_rewards, traj_correct)):
        infra = traj_infra[ti] if traj_infra is not None else None
        phis = traj_phis[ti] if traj_phis is not None else None
        for tu, r in enumerate(kevin_turn_returns(rw, cr, gamma, credit_incorrect=credit_incorrect,
                                                  phis=phis, phi_weight=phi_weight)):
            if infra is not None and tu < len(infra) and infra[tu]:
                continue
            rets.append(r)
            idx.append((ti, tu))
    return rets, idx


def token_mean_logprob(seq_logprob: float, n_tokens: int) -> float:
    return seq_logprob / max(int(n_tokens), 1)


def group_reward_std(rewards: Sequence[float]) -> float:
    n = len(rewards)
    if n < 2:
        return 0.0
    mu = sum(rewards) / n
    return math.sqrt(sum((r - mu) ** 2 for r in rewards) / n)


def starpo_keep_group(rewards, min_std: float = 1e-3) -> bool:
    return group_reward_std(rewards) > min_std


def starpo_select_high_variance(groups, keep_frac: float = 0.75, min_std: float = 1e-3) -> List[int]:
    """Indices (ascending) of the top ``keep_frac`` non-collapsed groups by std."""
    live = [(i, group_reward_std(g)) for i, g in enumerate(groups) if starpo_keep_group(g, min_std)]
    if not live:
        return []
    live.sort(key=lambda p: p[1], reverse=True)
    k = max(1, int(round(keep_frac * len(live))))
    return sorted(i for i, _ in live[:k])


def dynamic_sampling_refill(roll_fn: Callable[[int], object], target_groups: int, *,
                            min_std: float = 1e-3, max_attempts: int = 0, dynamic: bool = True,
                            std_key=None):
    """Roll groups until ``target_groups`` non-degenerate ones are kept (at most
    ``max_attempts`` rolls, default 3x target). Returns (kept, attempts)."""
    std_key = std_key or group_reward_std
    if max_attempts <= 0:
        max_attempts = 3 * target_groups if dynamic else target_groups
    kept, attempts = [], 0
    while len(kept) < target_groups and attempts < max_attempts:
        g = roll_fn(attempts)
        attempts += 1
        if dynamic and std_key(g) <= min_std:
            continue
        kept.append(g)
    return kept, attempts


def kl_k3(logp: float, ref_logp: float) -> float:
    """Schulman's k3 estimator exp(d) - d - 1 with d = ref - logp."""
    d = ref_logp - logp
    return math.exp(d) - d - 1.0


def value_prefilter(candidates: list, scorer, k: int) -> List[int]:
    if k >= len(candidates):
        return list(range(len(candidates)))
    order = sorted(range(len(candidates)), key=lambda i: scorer(candidates[i]), reverse=True)
    return sorted(order[:k])


def merge_across_ranks(per_rank: list) -> list:
    return [x for chunk in per_rank for x in chunk]


def distributed_group_advantages(per_rank_returns, variance_floor: float = 0.0,
                                 avspo_virtual_k: int = 2, adv_eps: float = EPS):
    """Normalise the full (all-rank) group once, then split back per rank."""
    flat = merge_across_ranks(per_rank_returns)
    adv = avspo_advantages(flat, variance_floor, avspo_virtual_k, adv_eps)
    out, i = [], 0
    for chunk in per_rank_returns:
        out.append(adv[i:i + len(chunk)])
        i += len(chunk)
    return out


def rank_slice(n: int, rank: int, world: int) -> List[int]:
    """Strided ownership: rank r gets r, r+world, ..."""
    return list(range(rank, n, max(1, world)))


# ----------------------------------------------------- GRPO -> token coefficients
@dataclass
class GRPOSample:
    """One trainable per-turn sample. ``logp``-type fields are token means."""
    adv: float
    n_tokens: int
    old_logp: Optional[float] = None
    ref_logp: Optional[float] = None
    sc_weight: Optional[float] = None


def grpo_sample_term(lp: float, s: GRPOSample, *, clip_lo: float, clip_hi: float,
                     ref_coef: float) -> Tuple[float, float]:
    """Value and derivative (w.r.t. the token-mean log-prob ``lp``) of one
    sample's GRPO term: -min(rA, clip(r)A) [* sc_w] + c*(e^d - d - 1)."""
    A = s.adv
    if s.old_logp is not None:
        r = math.exp(lp - s.old_logp)
        rc = min(max(r, 1 - clip_lo), 1 + clip_hi)
        if r * A <= rc * A:      # unclipped branch is the min
            pg, dpg = -r * A, -r * A
        else:                    # clipped branch: constant in lp
            pg, dpg = -rc * A, 0.0
    else:
        pg, dpg = -A * lp, -A
    if s.sc_weight is not None:
        pg, dpg = pg * s.sc_weight, dpg * s.sc_weight
    val, der = pg, dpg
    if ref_coef and s.ref_logp is not None:
        d = s.ref_logp - lp
        val += ref_coef * (math.exp(d) - d - 1.0)
        der += ref_coef * (1.0 - math.exp(d))
    return val, der


def grpo_token_coefficients(samples: Sequence[GRPOSample], lps: Sequence[float], *,
                            clip_lo: float, clip_hi: float, ref_coef: float,
                            total_tokens: int) -> Tuple[float, List[float]]:
    """Global token-mean GRPO loss = sum_s n_s * term_s / total_tokens.

    Returns (loss, per-sample coefficient c_s) such that every token of
    sample s gets dL/dlogp_t = c_s (the token mean spreads d/dlp over n_s
    tokens, which cancels the n_s weight)."""
    loss = 0.0
    coefs = []
    for s, lp in zip(samples, lps):
        v, d = grpo_sample_term(lp, s, clip_lo=clip_lo, clip_hi=clip_hi, ref_coef=ref_coef)
        loss += v * s.n_tokens / total_tokens
        coefs.append(d / total_tokens)
    return loss, coefs


# Anti-collapse pieces live in their own module; re-exported for existing callers.
from .anticollapse import (HIGH_REWARD_TOKEN, LOW_REWARD_TOKEN, DynamicStepController,  # noqa: E402,F401
                           avspo_advantages, code_shingle_cosine, gtpo_codesim_shaping,
                           prepend_reward_token, sample_reward_tokens, scgrpo_weight_from_kl,
                           variance_floor)
