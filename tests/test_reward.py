"""Reward ladder, physics reward, scanner, rooflines and config invariants (CPU)."""
import pytest

from kore_b200.analysis import rooflines as R
from kore_b200.config import CONFIG, KoreConfig
from kore_b200.policy.format import check_change_consistency, parse_response
from kore_b200.reward import stats
from kore_b200.reward.physics import PhysicsSignal, compute_residual_reward, residual_descent_frac
from kore_b200.reward.reward import (Observation, aggregate_speedup, compute_reward,
                                     roofline_ceiling_violation, scan_for_hacks)
from kore_b200.reward.timing_integrity import uncovered


def _ok(**kw):
    base = dict(compiled=True, validation_passed=True, snr_by_shape={"a": 40.0, "b": 35.0},
                wall_by_shape={"a": 1.0, "b": 2.0}, baseline_by_shape={"a": 1.5, "b": 2.0}, cv_pct=1.0)
    base.update(kw)
    return Observation(**base)


def test_tier_ordering():
    hack = compute_reward(Observation(compiled=True), source="import flashinfer\n")
    cf = compute_reward(Observation(compiled=False))
    inc = compute_reward(Observation(compiled=True, snr_db=20.0))
    ok = compute_reward(_ok())
    assert hack.tier == "hack" and cf.tier == "compile_fail" and inc.tier == "incorrect"
    assert hack.reward < cf.reward < inc.reward < CONFIG.correctness_weight <= ok.reward
    assert ok.speedup == pytest.approx(1.0)  # worst shape


def test_fast_p_bonus_and_excessive():
    r = compute_reward(_ok(baseline_by_shape={"a": 1.6, "b": 3.2}))
    assert "fast_p>=1.5" in r.flags
    r = compute_reward(_ok(baseline_by_shape={"a": 100.0, "b": 200.0}))
    assert "excessive_speedup" in r.flags and not any(f.startswith("fast_p") for f in r.flags)
    noisy = compute_reward(_ok(baseline_by_shape={"a": 1.6, "b": 3.2}, cv_pct=10.0))
    assert "high_variance" in noisy.flags


def test_aggregation_modes():
    obs = _ok(baseline_by_shape={"a": 1.0, "b": 8.0})
    cfg = KoreConfig(speed_aggregation="mean")
    assert aggregate_speedup(obs, cfg) == pytest.approx(2.0)
    assert aggregate_speedup(obs, KoreConfig()) == pytest.approx(1.0)


def test_scanner():
    assert scan_for_hacks("y = torch.matmul(a, b)")
    assert scan_for_hacks("import ctypes")
    assert scan_for_hacks("c = a @ b")
    assert scan_for_hacks("print('SNR: 99')")
    assert scan_for_hacks("# cublasGemmEx mentioned in a comment\nx = 1") is None
    assert scan_for_hacks('"""uses torch.matmul in docs"""\n@triton.jit\ndef k(x): pass') is None


def test_roofline_gate_and_physics():
    assert roofline_ceiling_violation(0.5, 1.0, 0.25)
    assert not roofline_ceiling_violation(None, 1.0)
    r = compute_reward(_ok(), roofline_gate=True, t_min_ms=5.0)
    assert r.tier == "hack" and "roofline_ceiling" in r.flags
    rho, pmc = residual_descent_frac(PhysicsSignal(t_min_ms=1.0, measured_ms=2.0))
    assert rho == pytest.approx(0.5) and not pmc
    rho2, pmc2 = residual_descent_frac(PhysicsSignal(1.0, 2.0, stall_frac=0.2, occupancy=0.9))
    assert pmc2 and rho2 >= rho
    rr = compute_residual_reward(_ok(), PhysicsSignal(1.0, 2.0))
    assert rr.tier == "correct_residual"


def test_config_invariants():
    with pytest.raises(ValueError):
        KoreConfig(eps_shape=0.3)
    with pytest.raises(ValueError):
        KoreConfig(reward_hack=0.5)
    assert CONFIG.snr_threshold_for("bf16") == CONFIG.snr_threshold_lowp


def test_rooflines_b200():
    p = R.resolve_peaks("sm_100a", use_measured=False)
    rf = R.roofline("g", "gemm_bf16", "bf16", "", {"M": 8192, "N": 8192, "K": 8192}, p, "sm_100a")
    assert rf.bound == "compute" and rf.t_min_ms == pytest.approx(2 * 8192 ** 3 / 2.25e15 * 1e3)
    rn = R.roofline("n", "rmsnorm", "bf16", "", {"M": 4096, "N": 4096}, p, "sm_100a")
    assert rn.bound == "memory"
    assert R.flops_bytes("attention_prefill", {"B": 1, "H": 32, "S": 2048, "D": 128, "KV": 8}, "bf16")
    assert R.fused_collective_roofline(1e12, 1e9, p) > 0


def test_stats_and_timing_coverage():
    assert stats.median([3, 1, 2]) == 2 and stats.median([1, 2, 3, 4]) == 2.5
    assert stats.cv_pct([1.0, 1.0]) == 0.0
    assert uncovered() == []


def test_parse_response_and_consistency():
    txt = ("<think>draft ```python\nbad\n```</think>\nANALYSIS: slow\nPROPOSED_CHANGE: BLOCK_M=128\n"
           "FULL_KERNEL:\n```python\nBLOCK_M = 128\n```")
    p = parse_response(txt)
    assert p["kernel"] == "BLOCK_M = 128" and p["analysis"] == "slow" and "draft" in p["think"]
    c = check_change_consistency("raise BLOCK_M", "BLOCK_M = 64", "BLOCK_M = 64", "BLOCK_M=128")
    assert not c["consistent"]
