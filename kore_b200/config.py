"""Central configuration of the verifier and reward (B200 target).

Same knobs as the reference's ``KoreConfig`` (kore/config.py:27-213) with the
hardware retargeted to sm_100a: the GPU target defaults to ``sm_100a`` and the
fp8 dtype is OCP e4m3. The reward-ladder invariants are asserted at
construction so an override can never invert a tier:

  reward_hack < reward_compile_fail < reward_incorrect,
  eps_shape + format_weight < correctness_weight,
  profile_reward_weight < smallest fast_p bonus.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
DATA_DIR = Path(os.environ.get("KORE_DATA_DIR", REPO_ROOT / "data"))
RUNS_DIR = Path(os.environ.get("KORE_RUNS_DIR", REPO_ROOT / "runs"))
CONFIGS_DIR = REPO_ROOT / "configs"


def _env(name, default, cast=str):
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    return cast(v)


@dataclass
class KoreConfig:
    gpu_target: str = field(default_factory=lambda: _env("GPU_TARGET", "sm_100a"))
    cuda_path: str = field(default_factory=lambda: _env("CUDA_HOME", "/usr/local/cuda"))
    # correctness gate
    snr_threshold_fp32: float = 30.0
    snr_threshold_lowp: float = 25.0
    atol: float = 1e-2
    rtol: float = 1e-2
    # benchmark trust
    warmup_iters: int = 10
    bench_iters: int = 30
    min_variance_runs: int = 3
    max_variance_runs: int = 5
    cv_threshold_pct: float = 3.0
    noise_floor_pct: float = 2.0
    l2_flush_bytes: int = 512 << 20          # > 2x the 126 MB L2 of a B200
    verifier_determinism_check: bool = True
    determinism_snr_tol_db: float = 10.0
    shape_augment: bool = field(default_factory=lambda: _env("KORE_SHAPE_AUGMENT", "0") == "1")
    shape_augment_max: int = 6
    # reward ladder
    correctness_weight: float = 0.3
    excessive_speedup_flag: float = 10.0
    reward_compile_fail: float = -1.0
    reward_incorrect: float = 0.0
    reward_hack: float = -1.5
    subthreshold_shaping: bool = True
    eps_shape: float = 0.05
    format_weight: float = 0.02
    reward_phase: str = "full"
    speedup_weight: float = 1.0
    speedup_log: bool = True
    fast_p_bonus: tuple = ((1.0, 0.30), (1.2, 0.30), (1.5, 0.40))
    fast_p_significant_only: bool = True
    profile_reward_weight: float = field(
        default_factory=lambda: _env("KORE_PROFILE_REWARD_WEIGHT", 0.0, float))
    speed_aggregation: str = field(default_factory=lambda: _env("KORE_SPEED_AGG", "worst"))
    cvar_alpha: float = 0.5
    gamma: float = 0.4
    data_dir: Path = DATA_DIR
    runs_dir: Path = RUNS_DIR

    def snr_threshold_for(self, dtype: str) -> float:
        """Relaxed floor for low-precision dtypes (their quantisation error is
        shared by candidate and oracle), strict fp32 floor otherwise."""
        d = (dtype or "").lower()
        low = ("fp8", "fp4", "fp6", "int8", "mxfp", "fp16", "bf16", "float16", "bfloat16")
        return self.snr_threshold_lowp if any(t in d for t in low) else self.snr_threshold_fp32

    def fp8_dtype(self):
        import torch
        return torch.float8_e4m3fn  # OCP e4m3 on Blackwell

    def __post_init__(self) -> None:
        self.check_invariants()

    def ensure_dirs(self) -> None:
        Path(self.data_dir).mkdir(parents=True, exist_ok=True)
        Path(self.runs_dir).mkdir(parents=True, exist_ok=True)

    def check_invariants(self) -> None:
        if self.speed_aggregation.lower() not in ("worst", "mean", "cvar"):
            raise ValueError(f"speed_aggregation must be worst|mean|cvar, got {self.speed_aggregation!r}")
        if not (0.0 < self.cvar_alpha <= 1.0):
            raise ValueError("cvar_alpha must be in (0, 1]")
        if not (self.reward_hack < self.reward_compile_fail < self.reward_incorrect):
            raise ValueError("need reward_hack < reward_compile_fail < reward_incorrect")
        if not (self.eps_shape + self.format_weight < self.correctness_weight):
            raise ValueError("eps_shape + format_weight must stay below correctness_weight")
        if self.profile_reward_weight and self.fast_p_bonus:
            if not self.profile_reward_weight < min(b for _, b in self.fast_p_bonus):
                raise ValueError("profile_reward_weight must be below the smallest fast_p bonus")


CONFIG = KoreConfig()
