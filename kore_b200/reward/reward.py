"""Lexicographic, hack-resistant kernel reward.

Tiers, each strictly dominating the ones below it:

    hack (-1.5) < compile_fail (-1) < incorrect (0 + bounded shaping)
        < correct (0.3 + speed term)

The speed term is scored on a distributionally robust aggregate of the
per-shape speedups against the vendor baseline (worst shape by default,
CVaR or geometric mean optionally), log-shaped above 1x, with cumulative
significance-gated bonuses at 1.0x / 1.2x / 1.5x; excessive speedups are
capped and high-variance timings damped. An optional roofline ceiling sends
physically impossible (faster than speed-of-light) timings to the hack tier.

Behavioural parity: kore/reward/reward.py:49-580. The delegation scanner is
retargeted to the CUDA/B200 stack: calls into cuBLAS/cuBLASLt/cuDNN,
CUTLASS, flashinfer, flash_attn, vLLM kernels or torch ops count as
delegation; so do escapes (subprocess, ctypes, exec, environment reads,
sleep) and forged verdict lines.
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional

from ..config import CONFIG
from ..obs import get_logger

_LOG = get_logger("reward")
DEFAULT_ROOFLINE_TOL = 0.25


@dataclass
class Observation:
    compiled: bool
    snr_db: Optional[float] = None
    wall_ms: Optional[float] = None
    baseline_ms: Optional[float] = None
    wall_by_shape: Dict[str, float] = field(default_factory=dict)
    baseline_by_shape: Dict[str, float] = field(default_factory=dict)
    snr_by_shape: Dict[str, float] = field(default_factory=dict)
    validation_passed: bool = False
    error_text: Optional[str] = None
    dtype: str = "fp32"
    cv_pct: Optional[float] = None
    flagged_hack: bool = False
    hack_reason: Optional[str] = None
    infra_error: bool = False
    profile_efficiency: Optional[float] = None
    counters: Optional[dict] = None


@dataclass
class RewardResult:
    reward: float
    correct: bool
    speedup: Optional[float]
    tier: str
    flags: List[str] = field(default_factory=list)
    detail: str = ""


# (regex, reason). Comments/docstrings are stripped before scanning.
_DELEGATION = [
    (r"\bcublas\w*|\bcublasLt\w*|\bcudnn\w*|\bcusparse\w*|\bcusolver\w*",
     "calls a CUDA vendor library instead of computing"),
    (r"\b(?:import|from)\s+(?:flashinfer|flash_attn|vllm|xformers|cutlass|deep_gemm|transformer_engine)\b",
     "imports a vendor kernel library instead of computing"),
    (r"\b(?:flashinfer|flash_attn|vllm|xformers|transformer_engine|deep_gemm)\.",
     "calls a vendor kernel library instead of computing"),
    (r"torch\.(?:matmul|mm|bmm|addmm|baddbmm|einsum|softmax|log_softmax|rms_norm|layer_norm|"
     r"scaled_dot_product_attention|tensordot|chain_matmul|mv|inner|vdot|dot|kron|conv\w*)\s*\(",
     "delegates to a torch op instead of a kernel"),
    (r"torch\.linalg\.\w+\s*\(", "delegates to torch.linalg"),
    (r"torch\.nn\.functional\.\w+\s*\(|\bF\.\w+\s*\(", "delegates to torch.nn.functional"),
    (r"torch\._C\b|torch\.ops\.\w+", "reaches torch internals / registered ops"),
    (r"\b(?!tl\.)(?!triton\.)[A-Za-z_]\w*\.(?:matmul|mm|bmm|addmm|baddbmm|einsum|"
     r"scaled_dot_product_attention|softmax|log_softmax|layer_norm|rms_norm|linear|conv\w*)\s*\(",
     "delegates an op through a handle"),
    (r"[\w\)\]][^\S\n]*@=?[^\S\n]*[\w\(]", "uses the @ matmul operator (vendor GEMM)"),
    (r"\bfrom\s+torch(?:\.\w+)*\s+import\b|\bimport\s+torch(?:\.\w+)*\s+as\s+\w+",
     "imports torch ops directly (delegation channel)"),
    (r"getattr\s*\(\s*(?:torch|np|numpy|F|nn|__builtins__|builtins)\b",
     "dynamic getattr on a numeric library"),
    (r"\b(?:import\s+reference|from\s+reference\s+import|from\s+[\w.]*\breference\b\s+import)\b",
     "imports the reference oracle"),
    (r"\b(?:reference|ref_program|ref_impl|\w+_oracle|oracle|ref_fn|baseline_fn)\s*\(",
     "calls the reference oracle / baseline instead of computing"),
    (r"\b(?:import\s+kore\w*|from\s+kore\w*)\b", "imports the framework to reach the oracle"),
    (r"\b(?:import|from)\s+(?:driver|reference)\b", "imports the sibling driver/reference"),
    (r"\bimportlib\b|__import__\s*\(|\bexec\s*\(|\beval\s*\(|\bcompile\s*\(",
     "dynamic import / exec escape"),
    (r"\bctypes\b|\bcffi\b|\bCDLL\b|dlopen|LoadLibrary|cuda\.bindings|\bcupy\b",
     "loads native code through a foreign-function interface"),
    (r"(?:SNR|allclose|median_ms|wall_ms|max_diff)\s*:", "prints a forged verifier verdict line"),
    (r"\bsys\.argv\b|\bargparse\b|\bgetopt\b", "reads the driver command line (mode sniffing)"),
    (r"['\"]--?(?:bench[-_]?mode|impl|warmup|iters|reference|candidate)['\"]",
     "references the driver's benchmark flags (mode sniffing)"),
    (r"\btime\.sleep\s*\(|\basyncio\.sleep\s*\(|__nanosleep", "sleeps (timing manipulation)"),
    (r"cudaProfilerStart|cudaDeviceSetLimit|set_sync_debug_mode|cudaSetDeviceFlags|"
     r"nvmlDeviceSet\w+|cudaGraphLaunch", "tampers with device / timing state"),
    (r"\bsubprocess\b|\bmultiprocessing\b|\bthreading\b|os\.system|os\.popen|os\.fork",
     "spawns processes or threads (isolation escape)"),
    (r"open\s*\([^)]*['\"][waxr]?[wax]\+?['\"]|\.write_text\s*\(|\.write_bytes\s*\(",
     "writes a file (filesystem escape)"),
    (r"\bos\.(?:chmod|replace|rename|remove|unlink|spawn\w*|posix_spawn)\b",
     "mutates the filesystem"),
    (r"\bsys\.modules\b", "reaches libraries through sys.modules"),
    (r"\bos\.environ\b|\bos\.getenv\b|\bgetenv\s*\(", "reads the environment"),
    (r"\batexit\b|signal\.signal|\bfaulthandler\b|sys\.excepthook|def\s+__del__\b",
     "registers an exit / signal hook (post-verdict forgery)"),
]
_COMPILED = [(re.compile(p), r) for p, r in _DELEGATION]
_SILENT_EXCEPT = re.compile(r"except\s*[\w. ,()]*:\s*(?:\n\s*)*(?:return|pass|out\s*=)", re.MULTILINE)


def strip_comments_and_docstrings(src: str) -> str:
    src = re.sub(r'"""[\s\S]*?"""', " ", src)
    src = re.sub(r"'''[\s\S]*?'''", " ", src)
    src = re.sub(r"(?m)#(?!include|define|pragma|if|endif|else|undef).*$", "", src)
    src = re.sub(r"//.*", "", src)
    src = re.sub(r"/\*[\s\S]*?\*/", " ", src)
    return src


def scan_for_hacks(source: str) -> Optional[str]:
    """A reason string when the candidate source delegates, escapes or forges."""
    code = strip_comments_and_docstrings(source or "")
    for pat, reason in _COMPILED:
        if pat.search(code):
            return reason
    if _SILENT_EXCEPT.search(code):
        return "silent except-fallback that can mask incorrect results"
    return None


def roofline_ceiling_violation(measured_ms, t_min_ms, tol: float = DEFAULT_ROOFLINE_TOL) -> bool:
    """measured < T_min * (1 - tol): faster than physically possible. Fails open
    (False) on missing/invalid inputs or tol >= 1."""
    try:
        m, t = float(measured_ms), float(t_min_ms)
    except (TypeError, ValueError):
        return False
    if not (m > 0 and t > 0):
        return False
    return m < t * (1.0 - max(0.0, tol))


def _min_wall(obs: Observation) -> Optional[float]:
    vals = [v for v in (obs.wall_by_shape or {}).values() if v and v > 0]
    if vals:
        return min(vals)
    return obs.wall_ms if obs.wall_ms and obs.wall_ms > 0 else None


def shape_speedups(obs: Observation) -> List[float]:
    out = []
    for k, cand in (obs.wall_by_shape or {}).items():
        base = (obs.baseline_by_shape or {}).get(k)
        if base and cand and cand > 0:
            out.append(base / cand)
    return out


def worst_speedup(obs: Observation) -> Optional[float]:
    r = shape_speedups(obs)
    if r:
        return min(r)
    if obs.baseline_ms and obs.wall_ms and obs.wall_ms > 0:
        return obs.baseline_ms / obs.wall_ms
    return None


def aggregate_speedup(obs: Observation, cfg=CONFIG) -> Optional[float]:
    """worst | cvar (geomean of the worst ceil(alpha*N)) | mean (geomean of all)."""
    r = shape_speedups(obs)
    if not r:
        return worst_speedup(obs)
    mode = (getattr(cfg, "speed_aggregation", "worst") or "worst").lower()
    n = len(r)
    if mode == "worst" or n == 1:
        return min(r)
    k = n if mode == "mean" else max(1, min(n, math.ceil(float(getattr(cfg, "cvar_alpha", 0.5)) * n)))
    logs = sorted(math.log(x) for x in r)[:k]
    return math.exp(sum(logs) / k)


def _worst_snr(obs: Observation) -> Optional[float]:
    vals = [v for v in (obs.snr_by_shape or {}).values() if v is not None]
    return min(vals) if vals else obs.snr_db


def subthreshold_credit(obs: Observation, dtype: str, cfg=CONFIG, snr_threshold=None) -> float:
    """eps_shape * clamp(worst SNR / threshold, 0, 1) for compiled-but-wrong kernels."""
    if not getattr(cfg, "subthreshold_shaping", False) or cfg.eps_shape <= 0:
        return 0.0
    thr = snr_threshold if snr_threshold is not None else cfg.snr_threshold_for(dtype)
    snr = _worst_snr(obs)
    if snr is None or not thr or thr <= 0:
        return 0.0
    return cfg.eps_shape * min(1.0, max(0.0, snr / thr))


def format_component(response: Optional[str], cfg=CONFIG) -> float:
    """+format_weight when the raw response carries a parsable kernel, minus
    that when it does not, 0 when no response is given."""
    if response is None or cfg.format_weight <= 0:
        return 0.0
    from ..policy.format import parse_response
    return cfg.format_weight if (parse_response(response).get("kernel") or "").strip() else -cfg.format_weight


def speedup_term(su_scored: float, su_raw: float, obs: Observation, cfg, flags: List[str]) -> float:
    """Speed credit of a correct kernel.

    The curve is linear below 1x and logarithmic above it (so a 4x kernel is
    not paid twice a 2x one); on top sit the fast_p bonuses, each paid when
    the raw speedup clears its threshold by the timing-noise margin. With
    ``fast_p_significant_only`` the bonuses need a trusted measurement: CV at
    most ``cv_threshold_pct`` and no excessive-speedup flag."""
    w = float(cfg.speedup_weight)
    curve = (lambda s: 1.0 + math.log(s)) if cfg.speedup_log else (lambda s: s)
    base = w * (curve(su_scored) if su_scored > 1.0 else max(su_scored, 0.0))
    table = list(cfg.fast_p_bonus or ())
    if not table:
        return base
    noisy = obs.cv_pct is not None and obs.cv_pct > cfg.cv_threshold_pct
    if cfg.fast_p_significant_only and (noisy or "excessive_speedup" in flags):
        return base
    need = 1.0 + cfg.noise_floor_pct / 100.0
    earned = [(thr, float(b)) for thr, b in table if su_raw >= thr * need]
    flags.extend(f"fast_p>={thr}" for thr, _ in earned)
    return base + sum(b for _, b in earned)


def all_shapes_pass(obs: Observation, dtype: str, cfg=CONFIG, snr_threshold=None) -> bool:
    thr = snr_threshold if snr_threshold is not None else cfg.snr_threshold_for(dtype)
    if obs.snr_by_shape:
        return all(v is not None and v >= thr for v in obs.snr_by_shape.values())
    return obs.snr_db is not None and obs.snr_db >= thr


def _done(rr: RewardResult) -> RewardResult:
    _LOG.emit("INFO" if rr.tier == "hack" else "DEBUG", "reward",
               {"tier": rr.tier, "reward": round(rr.reward, 4), "correct": rr.correct,
                "speedup": None if rr.speedup is None else round(rr.speedup, 4),
                "flags": list(rr.flags), "detail": rr.detail}, kind="event")
    return rr


def compute_reward(obs: Observation, source: str = "", dtype: str = "fp32", mode: str = "eval",
                   cfg=CONFIG, snr_threshold: Optional[float] = None, phase: Optional[str] = None,
                   response: Optional[str] = None, roofline_gate: bool = False,
                   t_min_ms: Optional[float] = None,
                   roofline_tol: float = DEFAULT_ROOFLINE_TOL) -> RewardResult:
    flags: List[str] = []
    phase = (phase or cfg.reward_phase or "full").lower()
    if obs.infra_error:
        return _done(RewardResult(cfg.reward_incorrect, False, None, "infra", ["infra"],
                                  obs.error_text or "infrastructure error"))
    hack = obs.hack_reason or (scan_for_hacks(source) if source else None)
    ceiling = False
    if not hack and roofline_gate and t_min_ms is not None:
        m = _min_wall(obs)
        if roofline_ceiling_violation(m, t_min_ms, roofline_tol):
            ceiling = True
            hack = (f"measured {m:.4g} ms is below the roofline T_min {t_min_ms:.4g} ms "
                    f"(tol {roofline_tol:.2f}): impossible throughput, measurement exploit")
    if hack:
        return _done(RewardResult(cfg.reward_hack, False, None, "hack",
                                  ["hack"] + (["roofline_ceiling"] if ceiling else []), str(hack)))
    if not obs.compiled:
        return _done(RewardResult(cfg.reward_compile_fail, False, None, "compile_fail", ["compile_fail"],
                                  obs.error_text or "did not compile"))
    if not (obs.validation_passed and all_shapes_pass(obs, dtype, cfg, snr_threshold)):
        credit = subthreshold_credit(obs, dtype, cfg, snr_threshold)
        fmt = format_component(response, cfg)
        flags = ["incorrect"] + (["shaped"] if credit > 0 else [])
        detail = obs.error_text or "failed correctness/SNR"
        if credit or fmt:
            detail += f" (shaped +{credit:.4f}, format {fmt:+.4f})"
        return _done(RewardResult(cfg.reward_incorrect + credit + fmt, False, None, "incorrect",
                                  flags, detail))
    fmt = format_component(response, cfg)
    su = aggregate_speedup(obs, cfg)
    if su is None:
        return _done(RewardResult(cfg.correctness_weight + fmt, True, None, "correct_no_bench", flags,
                                  "correct; no timing"))
    scored = su
    if su >= cfg.excessive_speedup_flag:
        flags.append("excessive_speedup")
        scored = cfg.excessive_speedup_flag
    if obs.cv_pct is not None and obs.cv_pct > cfg.cv_threshold_pct:
        flags.append("high_variance")
        scored = min(scored, 1.0)
    if phase == "correctness":
        flags.append("phase:correctness")
        speed = 0.0
    else:
        speed = speedup_term(scored, su, obs, cfg, flags)
        if cfg.profile_reward_weight > 0 and obs.profile_efficiency is not None:
            p = cfg.profile_reward_weight * max(0.0, min(1.0, obs.profile_efficiency))
            speed += p
            flags.append(f"profile+{p:.3f}")
    return _done(RewardResult(cfg.correctness_weight + speed + fmt, True, su, "correct_timed", flags,
                              f"worst-shape speedup {su:.3f}x vs baseline"
                              + (" [correctness phase: speed zeroed]" if phase == "correctness" else "")))
