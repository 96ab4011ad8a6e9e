"""Anti-collapse ladder for GRPO as its own import surface: RC-GRPO reward
tokens and variance floor, AVSPO virtual-sample advantages, SC-GRPO KL
weight, GTPO code-shingle shaping, and the plateau step controller. The
math lives in :mod:`kore_b200.policy.rl_math`.
Reference parity: kore/policy/anticollapse.py:41-213, dynamic.py:21-51.
"""
from .rl_math import (DynamicStepController, avspo_advantages, code_shingle_cosine, gtpo_codesim_shaping,  # noqa: F401
                      prepend_reward_token, sample_reward_tokens, scgrpo_weight_from_kl, variance_floor)
