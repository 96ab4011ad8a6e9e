"""Physics residual-descent reward and the single reward dispatch.

For a correct kernel the speed term becomes an absolute, roofline-grounded
credit: rho = T_min / (T_min + N) with the named residual
N = (stall fraction + occupancy deficit) * T_meas clamped to [0, T_meas - T_min]
when ncu counters are available, else eta = T_min / T_meas (flagged
``no_pmc``). All hack / compile / correctness gating is delegated to
:func:`compute_reward`, so the tier order is unchanged. On B200 the counters
come from ``ncu`` (``smsp__average_warps_issue_stalled_*`` /
``sm__warps_active``) instead of rocprofv3.

Behavioural parity: kore/reward/physics.py:61-348.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional, Tuple

from ..config import CONFIG
from .reward import (DEFAULT_ROOFLINE_TOL, Observation, RewardResult, compute_reward,
                     format_component, roofline_ceiling_violation)

DEFAULT_PHYSICS_WEIGHT = 1.0


@dataclass
class PhysicsSignal:
    t_min_ms: float
    measured_ms: Optional[float] = None
    stall_frac: Optional[float] = None
    occupancy: Optional[float] = None


def named_residual_ms(measured_ms: float, sig: PhysicsSignal) -> Optional[float]:
    if sig.stall_frac is None and sig.occupancy is None:
        return None
    stall = max(0.0, sig.stall_frac or 0.0)
    deficit = max(0.0, 1.0 - (sig.occupancy if sig.occupancy is not None else 1.0))
    resid = max(measured_ms - sig.t_min_ms, 0.0) if sig.t_min_ms == sig.t_min_ms else measured_ms
    return min(max((stall + deficit) * measured_ms, 0.0), resid)


def residual_descent_frac(sig: PhysicsSignal, measured_ms: Optional[float] = None) -> Tuple[Optional[float], bool]:
    t = sig.measured_ms if sig.measured_ms is not None else measured_ms
    if not t or t <= 0 or sig.t_min_ms is None or not sig.t_min_ms > 0:
        return None, False
    n = named_residual_ms(t, sig)
    if n is None:
        return min(sig.t_min_ms / t, 1.0), False
    return min(sig.t_min_ms / (sig.t_min_ms + n), 1.0), True


def compute_residual_reward(obs: Observation, physics: PhysicsSignal, source: str = "", dtype: str = "fp32",
                            cfg=CONFIG, physics_weight: float = DEFAULT_PHYSICS_WEIGHT,
                            snr_threshold=None, response=None, phase=None) -> RewardResult:
    base = compute_reward(obs, source=source, dtype=dtype, cfg=cfg, snr_threshold=snr_threshold,
                          response=response, phase=phase)
    if not base.correct:
        return base
    measured = obs.wall_ms
    if measured is None and obs.wall_by_shape:
        measured = max(obs.wall_by_shape.values())
    rho, pmc = residual_descent_frac(physics, measured)
    fmt = format_component(response, cfg)
    flags = list(base.flags)
    if rho is None:
        return RewardResult(cfg.correctness_weight + fmt, True, base.speedup, "correct_no_physics",
                            flags + ["no_physics"], "correct; no roofline/timing for residual credit")
    if not pmc:
        flags.append("no_pmc")
    return RewardResult(cfg.correctness_weight + physics_weight * max(rho, 0.0) + fmt, True, base.speedup,
                        "correct_residual", flags,
                        f"residual-descent rho={rho:.3f} ({'named-residual' if pmc else 'eta-fallback'}); "
                        f"credit={physics_weight * rho:.3f}")


def _walls(task, obs):
    walls = dict(getattr(obs, "wall_by_shape", None) or {})
    if not walls and getattr(obs, "wall_ms", None):
        prim = task.shape("primary") if hasattr(task, "shape") else None
        walls = {(prim.name if prim else "primary"): obs.wall_ms}
    return walls


def _shape_rooflines(task, obs, arch=None):
    from ..analysis.rooflines import detect_arch, resolve_peaks, roofline, shape_to_str
    a = arch or detect_arch()
    peaks = resolve_peaks(a)
    for name, wall in _walls(task, obs).items():
        if not wall or wall <= 0:
            continue
        sh = task.shape(name) if hasattr(task, "shape") else None
        dims = getattr(sh, "dims", None)
        if not dims:
            continue
        rf = roofline(task.task_id, task.operation, task.dtype, shape_to_str(dims), dims, peaks, a)
        if rf is not None and rf.t_min_ms > 0:
            yield name, wall, rf


def physics_signal_from_obs(task, obs, arch=None) -> Optional[PhysicsSignal]:
    """Worst-shape (minimum eta) physics signal from timings + rooflines."""
    worst = None
    for _, wall, rf in _shape_rooflines(task, obs, arch):
        e = rf.t_min_ms / wall
        if worst is None or e < worst[0]:
            worst = (e, rf.t_min_ms, wall)
    return None if worst is None else PhysicsSignal(t_min_ms=worst[1], measured_ms=worst[2])


def roofline_ceiling_violation_from_obs(task, obs, tol: float = DEFAULT_ROOFLINE_TOL, arch=None):
    for name, wall, rf in _shape_rooflines(task, obs, arch):
        if roofline_ceiling_violation(wall, rf.t_min_ms, tol):
            return True, (f"shape {name}: measured {wall:.4g} ms is below the roofline T_min "
                          f"{rf.t_min_ms:.4g} ms (tol {tol:.2f}): impossible throughput")
    return False, ""


def mask_reward_phase(rr: RewardResult, phase: str, correctness_weight: float) -> RewardResult:
    if str(phase).lower() == "correctness" and rr.correct:
        return replace(rr, reward=float(correctness_weight), speedup=None, tier="correct_masked")
    return rr


def compute_kernel_reward(obs: Observation, source: str, task, *, mode: str = "speedup", dtype: str = "fp32",
                          cfg=CONFIG, snr_threshold=None, physics_weight: float = DEFAULT_PHYSICS_WEIGHT,
                          response=None, reward_phase: str = "all", roofline_gate: bool = False,
                          roofline_tol: float = DEFAULT_ROOFLINE_TOL, arch=None) -> RewardResult:
    """One dispatch for the training loop: optional roofline ceiling gate, then
    residual (physics) or speedup reward, then the curriculum phase mask."""
    if roofline_gate:
        bad, why = roofline_ceiling_violation_from_obs(task, obs, roofline_tol, arch)
        if bad:
            return RewardResult(cfg.reward_hack, False, None, "hack", ["hack", "roofline_ceiling"], why)
    if mode == "residual":
        sig = physics_signal_from_obs(task, obs, arch)
        if sig is not None:
            rr = compute_residual_reward(obs, sig, source=source, dtype=dtype, cfg=cfg,
                                         physics_weight=physics_weight, snr_threshold=snr_threshold,
                                         response=response)
            return mask_reward_phase(rr, reward_phase, cfg.correctness_weight)
    rr = compute_reward(obs, source, dtype=dtype, cfg=cfg, snr_threshold=snr_threshold, response=response)
    return mask_reward_phase(rr, reward_phase, cfg.correctness_weight)
