"""Roofline-grounded ("physics") scoring of a correct kernel.

The speedup reward measures a candidate against a baseline that may itself be
far from the hardware limit. This module scores it against the limit instead:

* ``RooflineEvidence`` is what is known about one timed shape: the roofline
  time ``t_min`` (from the shape's FLOPs and bytes at the measured B200 peaks),
  the measured time ``t``, and optionally two ncu counters (issue-stall
  fraction, achieved occupancy).
* Its ``attainment`` is ``t_min / (t_min + N)``, where ``N`` is the part of the
  gap to the roofline that the counters can name: ``(stall + (1 - occupancy))
  * t``, clipped to ``[0, t - t_min]``. Without counters it degrades to
  ``eta = t_min / t``. This is the residual-descent formula of
  kore/reward/physics.py:77-113; it is what makes the credit grow when a
  kernel removes a stall even before its wall time moves.
* ``KernelScorer`` is the single entry the GRPO environment calls. Its order
  is: roofline ceiling gate (a time below ``t_min`` beyond a tolerance is a
  measurement exploit and scores as a hack), then the ladder of
  :func:`compute_reward` for every non-correct outcome, then the physics credit
  (``mode="residual"``) or the speedup credit (``mode="speedup"``), and finally
  the curriculum phase mask (``"correctness"`` pays only the correctness
  weight). Reference dispatch: kore/reward/physics.py:296-348.

On B200 the counters come from ncu
(``smsp__average_warps_issue_stalled_*`` and ``sm__warps_active``).
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Iterator, Optional, Tuple

from ..config import CONFIG
from .reward import (DEFAULT_ROOFLINE_TOL, Observation, RewardResult, compute_reward,
                     format_component, roofline_ceiling_violation)

DEFAULT_PHYSICS_WEIGHT = 1.0


@dataclass
class RooflineEvidence:
    """Roofline time, measured time and optional counters of one shape (ms)."""
    t_min_ms: float
    measured_ms: Optional[float] = None
    stall_frac: Optional[float] = None
    occupancy: Optional[float] = None

    @property
    def has_counters(self) -> bool:
        return self.stall_frac is not None or self.occupancy is not None

    def residual_ms(self, t: float) -> Optional[float]:
        """The named part of the gap ``t - t_min`` (None without counters)."""
        if not self.has_counters:
            return None
        lost = max(0.0, self.stall_frac or 0.0)
        if self.occupancy is not None:
            lost += max(0.0, 1.0 - self.occupancy)
        gap = t - self.t_min_ms if self.t_min_ms == self.t_min_ms else t
        return max(0.0, min(lost * t, max(gap, 0.0)))

    def attainment(self, measured_ms: Optional[float] = None) -> Tuple[Optional[float], bool]:
        """(score in [0, 1], whether counters named the residual)."""
        t = self.measured_ms if self.measured_ms is not None else measured_ms
        if t is None or t <= 0 or self.t_min_ms is None or not self.t_min_ms > 0:
            return None, False
        n = self.residual_ms(t)
        if n is None:
            return min(1.0, self.t_min_ms / t), False
        return min(1.0, self.t_min_ms / (self.t_min_ms + n)), True


# Older name kept for callers that construct the signal directly.
PhysicsSignal = RooflineEvidence


def residual_descent_frac(ev: RooflineEvidence, measured_ms: Optional[float] = None):
    return ev.attainment(measured_ms)


def _timed_shapes(task, obs) -> Iterator[Tuple[str, float]]:
    walls = dict(getattr(obs, "wall_by_shape", None) or {})
    if not walls and getattr(obs, "wall_ms", None):
        prim = task.shape("primary") if hasattr(task, "shape") else None
        walls = {prim.name if prim is not None else "primary": obs.wall_ms}
    for name, wall in walls.items():
        if wall and wall > 0:
            yield name, wall


class KernelScorer:
    """Scores one verified kernel; configured once per GRPO run."""

    def __init__(self, *, mode: str = "speedup", cfg=CONFIG, physics_weight: float = DEFAULT_PHYSICS_WEIGHT,
                 reward_phase: str = "all", roofline_gate: bool = False,
                 roofline_tol: float = DEFAULT_ROOFLINE_TOL, arch: Optional[str] = None):
        if mode not in ("speedup", "residual"):
            raise ValueError(f"reward mode must be speedup|residual, got {mode!r}")
        self.mode = mode
        self.cfg = cfg
        self.weight = physics_weight
        self.phase = str(reward_phase or "all").lower()
        self.gate = roofline_gate
        self.tol = roofline_tol
        self.arch = arch

    # -- roofline per shape
    def rooflines(self, task, obs):
        from ..analysis.rooflines import detect_arch, resolve_peaks, roofline, shape_to_str
        arch = self.arch or detect_arch()
        peaks = resolve_peaks(arch)
        for name, wall in _timed_shapes(task, obs):
            sh = task.shape(name) if hasattr(task, "shape") else None
            dims = getattr(sh, "dims", None)
            if not dims:
                continue
            rf = roofline(task.task_id, task.operation, task.dtype, shape_to_str(dims), dims, peaks, arch)
            if rf is not None and rf.t_min_ms > 0:
                yield name, wall, rf.t_min_ms

    def evidence(self, task, obs) -> Optional[RooflineEvidence]:
        """The evidence of the shape furthest from its roofline."""
        worst = min(((t_min / wall, t_min, wall) for _, wall, t_min in self.rooflines(task, obs)),
                    default=None)
        return None if worst is None else RooflineEvidence(t_min_ms=worst[1], measured_ms=worst[2])

    def ceiling_breach(self, task, obs) -> Optional[str]:
        for name, wall, t_min in self.rooflines(task, obs):
            if roofline_ceiling_violation(wall, t_min, self.tol):
                return (f"shape {name}: {wall:.4g} ms beats the roofline minimum {t_min:.4g} ms by more "
                        f"than the {self.tol:.0%} tolerance, which no kernel can do")
        return None

    # -- credit
    def physics_credit(self, obs: Observation, ev: RooflineEvidence, base: RewardResult,
                       response: Optional[str]) -> RewardResult:
        t = obs.wall_ms
        if t is None and obs.wall_by_shape:
            t = max(obs.wall_by_shape.values())
        score, named = ev.attainment(t)
        fmt = format_component(response, self.cfg)
        if score is None:
            return RewardResult(self.cfg.correctness_weight + fmt, True, base.speedup, "correct_no_physics",
                                list(base.flags) + ["no_physics"], "correct, but no roofline time to score")
        flags = list(base.flags) + ([] if named else ["no_pmc"])
        credit = self.weight * max(score, 0.0)
        how = "counter-named residual" if named else "eta (no counters)"
        return RewardResult(self.cfg.correctness_weight + credit + fmt, True, base.speedup,
                            "correct_residual", flags, f"roofline attainment {score:.3f} by {how}, "
                            f"credit {credit:.3f}")

    def _mask(self, rr: RewardResult) -> RewardResult:
        if self.phase == "correctness" and rr.correct:
            return replace(rr, reward=float(self.cfg.correctness_weight), speedup=None, tier="correct_masked")
        return rr

    def score(self, obs: Observation, source: str, task, *, dtype: str = "fp32",
              snr_threshold=None, response: Optional[str] = None,
              evidence: Optional[RooflineEvidence] = None) -> RewardResult:
        if self.gate:
            why = self.ceiling_breach(task, obs)
            if why:
                return RewardResult(self.cfg.reward_hack, False, None, "hack", ["hack", "roofline_ceiling"], why)
        base = compute_reward(obs, source, dtype=dtype, cfg=self.cfg, snr_threshold=snr_threshold,
                              response=response)
        if self.mode == "residual" and base.correct:
            ev = evidence if evidence is not None else self.evidence(task, obs)
            if ev is not None:
                base = self.physics_credit(obs, ev, base, response)
        return self._mask(base)


def compute_residual_reward(obs: Observation, evidence: RooflineEvidence, source: str = "",
                            dtype: str = "fp32", cfg=CONFIG,
                            physics_weight: float = DEFAULT_PHYSICS_WEIGHT, snr_threshold=None,
                            response=None, phase=None) -> RewardResult:
    """Residual-mode score of an observation whose roofline evidence is already known."""
    sc = KernelScorer(mode="residual", cfg=cfg, physics_weight=physics_weight)
    base = compute_reward(obs, source=source, dtype=dtype, cfg=cfg, snr_threshold=snr_threshold,
                          response=response, phase=phase)
    return sc.physics_credit(obs, evidence, base, response) if base.correct else base


def physics_signal_from_obs(task, obs, arch=None) -> Optional[RooflineEvidence]:
    return KernelScorer(arch=arch).evidence(task, obs)


def compute_kernel_reward(obs: Observation, source: str, task, *, mode: str = "speedup", dtype: str = "fp32",
                          cfg=CONFIG, snr_threshold=None, physics_weight: float = DEFAULT_PHYSICS_WEIGHT,
                          response=None, reward_phase: str = "all", roofline_gate: bool = False,
                          roofline_tol: float = DEFAULT_ROOFLINE_TOL, arch=None) -> RewardResult:
    """Functional form of ``KernelScorer(...).score(...)``."""
    return KernelScorer(mode=mode, cfg=cfg, physics_weight=physics_weight, reward_phase=reward_phase,
                        roofline_gate=roofline_gate, roofline_tol=roofline_tol, arch=arch
                        ).score(obs, source, task, dtype=dtype, snr_threshold=snr_threshold, response=response)
