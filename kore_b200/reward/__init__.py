"""Kernel reward: lexicographic ladder, physics (roofline residual) reward,
potential-based shaping, ncu-counter dense terms, timing statistics."""
from .reward import Observation, RewardResult, compute_reward, scan_for_hacks  # noqa: F401
