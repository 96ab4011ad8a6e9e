"""Potential-based reward shaping (Ng, Harada & Russell, 1999).

F_t = gamma * Phi(s_{t+1}) - Phi(s_t) with ``phis[t]`` the potential of the
state ENTERING turn t and ``terminal_phi`` past the last turn; the discounted
sum telescopes to -Phi(s_0). A ``None`` potential on either side makes that
transition's term 0. Behavioural parity: kore/reward/shaping.py:50-103.
"""
from __future__ import annotations

from typing import List, Optional, Sequence


def shaping_terms(phis: Sequence[Optional[float]], gamma: float, terminal_phi: float = 0.0) -> List[float]:
    out = []
    for t, cur in enumerate(phis):
        nxt = phis[t + 1] if t + 1 < len(phis) else terminal_phi
        out.append(0.0 if cur is None or nxt is None else gamma * float(nxt) - float(cur))
    return out


def shaped_turn_rewards(turn_rewards: Sequence[float], phis: Sequence[Optional[float]], gamma: float,
                        weight: float = 1.0, terminal_phi: float = 0.0) -> List[float]:
    if len(turn_rewards) != len(phis):
        raise ValueError(f"turn_rewards ({len(turn_rewards)}) and phis ({len(phis)}) differ in length")
    return [float(r) + weight * f for r, f in zip(turn_rewards, shaping_terms(phis, gamma, terminal_phi))]


def discounted_shaping_sum(phis: Sequence[Optional[float]], gamma: float, terminal_phi: float = 0.0) -> float:
    return float(sum(gamma ** t * f for t, f in enumerate(shaping_terms(phis, gamma, terminal_phi))))
