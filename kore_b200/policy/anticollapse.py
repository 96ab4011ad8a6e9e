"""Anti-collapse ladder of the GRPO trainer.

Group-relative advantages vanish when every member of a group scores the same
(all correct or all wrong); these pieces keep a learning signal alive:

* RC-GRPO: condition a share of each group's prompts on a high/low reward
  token and floor the variance when the two halves collapse
  (kore/policy/anticollapse.py:41-106).
* AVSPO: add ``k`` virtual samples at +-tau when the group std is below tau,
  so a uniform group still has a direction (kore/policy/anticollapse.py:108-136).
* SC-GRPO: down-weight samples whose token KL to the reference is large
  (kore/policy/anticollapse.py:139-175).
* GTPO: shape rewards by code similarity (token-shingle cosine) to known-good
  kernels (kore/policy/anticollapse.py:177-213).
* A plateau controller that stops a run whose reward stopped moving
  (kore/policy/dynamic.py:21-51).
"""
from __future__ import annotations

import math
import random
import re
from dataclasses import dataclass
from typing import List, Optional

EPS = 1e-6        # the group-advantage epsilon of rl_math (kept here so either module imports first)

HIGH_REWARD_TOKEN = "<|high_reward|>"
LOW_REWARD_TOKEN = "<|low_reward|>"


def prepend_reward_token(prompt: str, token: str) -> str:
    if token not in (HIGH_REWARD_TOKEN, LOW_REWARD_TOKEN):
        raise ValueError(f"unknown reward token {token!r}")
    return f"{token}\n{prompt}"


def sample_reward_tokens(G: int, p_high: float, seed: Optional[int] = None) -> List[str]:
    """Exactly round(G*p_high) high tokens, shuffled."""
    if G < 0:
        raise ValueError("G must be non-negative")
    n_high = min(G, max(0, int(round(G * min(1.0, max(0.0, p_high))))))
    toks = [HIGH_REWARD_TOKEN] * n_high + [LOW_REWARD_TOKEN] * (G - n_high)
    random.Random(seed).shuffle(toks)
    return toks


def variance_floor(rewards, reward_tokens, means: dict) -> bool:
    """RC-GRPO check: observed variance >= (G-1)/G * p(1-p) * gap^2."""
    G = len(rewards)
    if G == 0:
        return False
    p = sum(1 for t in reward_tokens if t == HIGH_REWARD_TOKEN) / G
    vals = [v for v in means.values() if v is not None]
    gap = (max(vals) - min(vals)) if len(vals) >= 2 else 0.0
    floor = (G - 1) / G * p * (1 - p) * gap * gap
    mu = sum(rewards) / G
    return sum((r - mu) ** 2 for r in rewards) / G >= floor


def avspo_advantages(returns, tau: float, k: int = 2, eps: float = EPS) -> List[float]:
    """Group advantages whose normaliser includes k virtual samples at
    mean +/- tau when the real std is below tau (mean unchanged)."""
    n = len(returns)
    if n == 0:
        return []
    mu = sum(returns) / n
    var = sum((r - mu) ** 2 for r in returns) / n
    sd = math.sqrt(var)
    if tau <= 0 or k <= 0 or sd >= tau:
        return [(r - mu) / (sd + eps) for r in returns]
    sd_aug = math.sqrt((n * var + k * tau * tau) / (n + k))
    return [(r - mu) / (sd_aug + eps) for r in returns]


def scgrpo_weight_from_kl(token_kls, scale: float = 1.0, w_min: float = 0.5,
                          w_max: float = 2.0) -> float:
    if not token_kls:
        return 1.0
    return max(w_min, min(w_max, 1.0 + scale * sum(token_kls) / len(token_kls)))


_TOK_RE = re.compile(r"[A-Za-z_]\w*|\d+|[^\s\w]")


def _shingles(code: str, n: int = 3) -> dict:
    toks = _TOK_RE.findall(code or "")
    if not toks:
        return {}
    n = max(1, min(n, len(toks)))
    out: dict = {}
    for i in range(len(toks) - n + 1):
        key = tuple(toks[i:i + n])
        out[key] = out.get(key, 0) + 1
    return out


def code_shingle_cosine(a: str, b: str, n: int = 3) -> float:
    ca, cb = _shingles(a, n), _shingles(b, n)
    if not ca or not cb:
        return 0.0
    dot = sum(v * cb.get(k, 0) for k, v in ca.items())
    na = math.sqrt(sum(v * v for v in ca.values()))
    nb = math.sqrt(sum(v * v for v in cb.values()))
    return dot / (na * nb) if na and nb else 0.0


def gtpo_codesim_shaping(codes, references, scale: float = 0.3, n: int = 3) -> List[float]:
    """All-fail groups: partial reward = scale * max cosine to any reference."""
    if not references:
        return [0.0] * len(codes)
    return [scale * max((code_shingle_cosine(c, r, n) for r in references), default=0.0)
            for c in codes]


# ---------------------------------------------------------------- plateau stop
@dataclass
class DynamicStepController:
    min_steps: int
    max_steps: int
    patience: int
    min_delta: float = 1e-3
    best: float = -math.inf
    best_step: int = -1
    stopped_reason: str = ""

    def update(self, step: int, metric: float) -> bool:
        """Record the metric of 0-based ``step``; True means stop."""
        if metric > self.best + self.min_delta:
            self.best, self.best_step = metric, step
        done = step + 1
        if done >= self.max_steps:
            self.stopped_reason = f"reached max_steps={self.max_steps}"
            return True
        if done < self.min_steps:
            return False
        if self.best_step >= 0 and step - self.best_step >= self.patience:
            self.stopped_reason = (f"plateau: no >{self.min_delta} gain for {self.patience} steps "
                                   f"(best={self.best:.4f} @ step {self.best_step})")
            return True
        return False
