"""Environment interface of the GRPO rollout loop + the synthetic benchmark env.

An environment renders a task's first prompt and scores each turn's
response. ``TurnResult`` carries the per-turn reward, the correctness flag
used by Kevin credit, the feedback text for the next turn, the potential Phi
of the resulting state (for potential-based shaping), and an infrastructure
flag (infra turns are dropped from training).
"""
from __future__ import annotations

import random
import zlib
from dataclasses import dataclass
from typing import Any, List, Optional


@dataclass
class TurnResult:
    reward: float
    correct: bool
    feedback: str = ""
    phi: Optional[float] = None
    infra: bool = False
    obs: Any = None
    code: str = ""


class RolloutEnv:
    """Base class: subclasses implement ``prompt_messages`` and ``step``."""

    def prompt_messages(self, task) -> List[dict]:
        raise NotImplementedError

    def step(self, task, response: str, turn: int, traj: int, history: List[TurnResult]) -> TurnResult:
        raise NotImplementedError


def stable_seed(*parts) -> int:
    """Process-independent seed (Python's hash() of str is salted per process)."""
    return zlib.crc32(repr(parts).encode()) & 0xFFFFFFFF


class SyntheticRewardEnv(RolloutEnv):
    """Benchmark env (BASELINE GRPO config): per-turn reward uniform in
    {0, 0.1, 0.3} plus the shaping term 0.9 * Phi' - Phi with Phi ~ U(0, 1),
    all drawn from a seed; every turn counts as correct so the trajectory
    credit is exercised. Prompts are uniform-random token ids."""

    def __init__(self, seed: int = 0, prompt_len: int = 1024, feedback_len: int = 32,
                 vocab_size: int = 151936, gamma_phi: float = 0.9):
        self.seed = seed
        self.prompt_len = prompt_len
        self.feedback_len = feedback_len
        self.vocab = vocab_size
        self.gamma_phi = gamma_phi

    def prompt_ids(self, task) -> List[int]:
        rng = random.Random(stable_seed(self.seed, "prompt", task))
        return [rng.randrange(self.vocab) for _ in range(self.prompt_len)]

    def feedback_ids(self, task, turn: int, traj: int) -> List[int]:
        rng = random.Random(stable_seed(self.seed, "fb", task, turn, traj))
        return [rng.randrange(self.vocab) for _ in range(self.feedback_len)]

    def step(self, task, response, turn, traj, history) -> TurnResult:
        rng = random.Random(stable_seed(self.seed, "r", task, turn, traj))
        r = rng.choice([0.0, 0.1, 0.3])
        phi_prev = history[-1].phi if history else rng.random()
        phi = rng.random()
        return TurnResult(reward=r + self.gamma_phi * phi - (phi_prev or 0.0), correct=True, phi=phi)
