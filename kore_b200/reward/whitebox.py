"""White-box potential Phi(s) from ncu counters of a candidate kernel.

stall fraction and achieved occupancy are read from Nsight Compute metric
names (the B200 replacement for rocprofv3's MemUnitStalled /
OccupancyPercent); Phi is the roofline attainment of the kernel, upgraded to
the named-residual rho when counters are present. Behavioural parity:
kore/reward/whitebox.py:71-188.
"""
from __future__ import annotations

from typing import Optional

from .physics import PhysicsSignal, physics_signal_from_obs, residual_descent_frac


def _clamp01(x):
    return None if x is None else max(0.0, min(1.0, float(x)))


def _lookup(counters: dict, *names):
    for n in names:
        if counters and n in counters and counters[n] is not None:
            try:
                return float(counters[n])
            except (TypeError, ValueError):
                continue
    return None


def stall_frac_from_counters(counters: dict) -> Optional[float]:
    """Fraction of issue slots lost to memory-side stalls (ncu percent or ratio)."""
    v = _lookup(counters, "stall_frac", "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
                "smsp__pcsamp_warps_issue_stalled_long_scoreboard.pct", "MemUnitStalled")
    if v is None:
        return None
    return _clamp01(v / 100.0 if v > 1.0 else v)


def occupancy_from_counters(counters: dict) -> Optional[float]:
    v = _lookup(counters, "occupancy", "sm__warps_active.avg.pct_of_peak_sustained_active",
                "OccupancyPercent")
    if v is None:
        return None
    return _clamp01(v / 100.0 if v > 1.0 else v)


def physics_signal_from_counters(task, obs, counters: Optional[dict], arch=None) -> Optional[PhysicsSignal]:
    sig = physics_signal_from_obs(task, obs, arch)
    if sig is None or not counters:
        return sig
    sig.stall_frac = stall_frac_from_counters(counters)
    sig.occupancy = occupancy_from_counters(counters)
    return sig


def whitebox_attainment(task, obs, counters=None, arch=None) -> Optional[float]:
    sig = physics_signal_from_counters(task, obs, counters, arch)
    if sig is None:
        return None
    rho, _ = residual_descent_frac(sig)
    return rho


def whitebox_structural_score(counters: dict, *, flops: Optional[float] = None,
                              bytes_: Optional[float] = None) -> Optional[float]:
    """Counter-only score in [0,1]: mean of (1 - stall) and occupancy, times the
    tensor-pipe activity when a contraction's counters are present."""
    s = stall_frac_from_counters(counters)
    o = occupancy_from_counters(counters)
    parts = [p for p in ((1.0 - s) if s is not None else None, o) if p is not None]
    if not parts:
        return None
    score = sum(parts) / len(parts)
    tc = _lookup(counters, "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active")
    if tc is not None and flops and bytes_ and flops / max(bytes_, 1.0) > 50:
        score *= _clamp01(tc / 100.0)
    return _clamp01(score)


def phi_potential(task, obs, counters: Optional[dict] = None, arch=None) -> Optional[float]:
    """Phi(s) for potential-based shaping; None for incorrect / untimed kernels."""
    if obs is None or not getattr(obs, "validation_passed", False):
        return None
    return whitebox_attainment(task, obs, counters, arch)
