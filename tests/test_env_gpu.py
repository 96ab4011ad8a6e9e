"""KoreEnv end to end on the GPU: seed kernels verify and time against the
vendor baseline, wrong kernels are caught, rewards follow the ladder."""
import pytest

from kore_b200.env.kore_env import KernelRolloutEnv, KoreEnv
from kore_b200.policy.configs import GRPOConfig
from kore_b200.reward.reward import compute_reward
from kore_b200.tasks.registry import get_task

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tid", ["rmsnorm_bf16", "silu_mul_bf16", "gen_add_bf16"])
def test_seed_kernels_pass_and_time(tid):
    t = get_task(tid)
    obs = KoreEnv(t, timeout_s=300).step(t.seed_src)
    assert obs.compiled and obs.validation_passed, obs.error_text
    assert obs.wall_ms and obs.wall_ms > 0 and obs.baseline_ms and obs.baseline_ms > 0
    rr = compute_reward(obs, t.seed_src, dtype=t.dtype)
    assert rr.correct and rr.reward >= 0.3


def test_wrong_kernel_is_incorrect():
    t = get_task("silu_mul_bf16")
    wrong = t.seed_src.replace("y = a / (1.0 + tl.exp(-a)) * b", "y = a * b")
    obs = KoreEnv(t, timeout_s=300).step(wrong)
    assert obs.compiled and not obs.validation_passed
    assert compute_reward(obs, wrong).tier == "incorrect"


def test_syntax_error_is_compile_fail():
    obs = KoreEnv("gen_add_bf16", timeout_s=120).step("def add(a, b):\n    return (\n")
    assert not obs.compiled


def test_rollout_env_turn():
    env = KernelRolloutEnv(GRPOConfig(reward_mode="residual"))
    t = get_task("gen_relu_bf16")
    resp = f"ANALYSIS: seed\nPROPOSED_CHANGE: none\nFULL_KERNEL:\n```python\n{t.seed_src}\n```"
    tr = env.step(t.task_id, resp, 0, 0, [])
    assert tr.correct and tr.reward > 0.3 and "CORRECT" in tr.feedback
