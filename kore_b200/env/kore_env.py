"""KoreEnv: the verified kernel environment (B200 target).

``KoreEnv(task).step(source) -> Observation``:
  1. hack scan of the candidate source (delegation / escape / forgery);
  2. replay-cache lookup;
  3. stage a private work dir: the candidate as ``kernel.py`` (task files are
     read-only 0o444);
  4. correctness: one driver subprocess per shape (new session, process group
     killed on timeout, rlimits), verdict parsed from the LAST matching lines;
     SNR gate per shape (dtype-aware threshold, or the task's override);
  5. determinism re-run of the primary shape (SNR must stay within a
     tolerance and still pass);
  6. timing under an exclusive per-GPU flock: one ``--bench-both`` process
     for all shapes (candidate and vendor baseline alternated, cold L2,
     randomised iteration counts), repeated until the CV is low enough; the
     candidate's output is re-verified after timing (poisoned-result check);
  7. optional ncu counters (``collect_counters``) of one candidate call and
     one vendor-baseline call (``--profile-run``, an NVTX-selected capture)
     for the white-box reward and the counter-relative profile score;
  8. cache the observation.
Failures are classified as compile / incorrect / infra (timeouts, OOM,
signals, CUDA errors, missing modules are infra and are never cached or
trained on). Reference parity: kore/env/kore_env.py:115-756.
"""
from __future__ import annotations

import fcntl
import os
import re
import resource
import shutil
import signal
import subprocess
import sys
import tempfile
import time
from contextlib import contextmanager
from typing import Dict, List, Optional

from ..config import CONFIG
from ..obs import get_logger
from ..reward.reward import Observation, scan_for_hacks
from ..reward.stats import median
from ..tasks.base import Task
from ..tasks.registry import get_task
from .base import RolloutEnv, TurnResult
from .replay import ReplayCache

log = get_logger("env.kore")
_INFRA = re.compile(r"out of memory|CUDA error|illegal memory|Killed|Segmentation fault|"
                    r"ModuleNotFoundError: No module named '(?!candidate)|cudaErrorLaunchFailure|"
                    r"device-side assert|NCCL error", re.IGNORECASE)
_SNR = re.compile(r"^SNR:\s*(-?[\d.]+|inf|-inf)", re.MULTILINE)
_ALLCLOSE = re.compile(r"^allclose:\s*(True|False)", re.MULTILINE)
_BENCH = re.compile(r"^(CAND|REF)\s+(\S+)\s+([\d.]+)\s+([\d.]+)", re.MULTILINE)
_POST = re.compile(r"^POST_VERIFY_SNR\s+(\S+)\s+(-?[\d.]+)", re.MULTILINE)


def _limit_child():
    os.setsid()
    try:
        resource.setrlimit(resource.RLIMIT_NPROC, (4096, 4096))
    except (ValueError, OSError):
        pass


class KoreEnv:
    def __init__(self, task, *, gpu: Optional[int] = None, timeout_s: float = 180.0,
                 cache: Optional[ReplayCache] = None, cfg=CONFIG, collect_pmc: bool = False,
                 python: Optional[str] = None):
        self.task: Task = task if isinstance(task, Task) else get_task(task)
        self.gpu = gpu
        self.timeout = timeout_s
        self.cache = cache
        self.cfg = cfg
        self.collect_pmc = collect_pmc
        self.python = python or sys.executable

    # ------------------------------------------------------------ process
    def _env(self) -> Dict[str, str]:
        env = dict(os.environ)
        if self.gpu is not None:
            env["CUDA_VISIBLE_DEVICES"] = str(self.gpu)
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        return env

    def _exec(self, args: List[str], cwd: str, timeout: Optional[float] = None):
        """Run the driver; returns (rc, stdout+stderr, timed_out)."""
        p = subprocess.Popen([self.python, "-m", "kore_b200.tasks.driver"] + args, cwd=cwd,
                             stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=self._env(),
                             preexec_fn=_limit_child)
        try:
            out, _ = p.communicate(timeout=timeout or self.timeout)
            return p.returncode, out, False
        except subprocess.TimeoutExpired:
            try:
                os.killpg(p.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            out, _ = p.communicate()
            return -9, out or "", True

    @contextmanager
    def _timing_lock(self):
        """Exclusive per-GPU lock so timings never overlap other benches."""
        path = os.path.join(tempfile.gettempdir(), f"kore_timing_gpu{self.gpu if self.gpu is not None else 0}.lock")
        with open(path, "w") as fh:
            fcntl.flock(fh, fcntl.LOCK_EX)
            try:
                yield
            finally:
                fcntl.flock(fh, fcntl.LOCK_UN)

    # ------------------------------------------------------------ steps
    def step(self, source: str) -> Observation:
        return self.evaluate(source)

    def evaluate(self, source: str) -> Observation:
        t = self.task
        hack = scan_for_hacks(source)
        if hack:
            return Observation(compiled=True, flagged_hack=True, hack_reason=hack, dtype=t.dtype)
        if self.cache is not None:
            hit = self.cache.get(t.task_id, source)
            if hit is not None:
                return hit
        obs = self._run(source)
        if self.cache is not None:
            self.cache.put(t.task_id, source, obs)
        return obs

    def _run(self, source: str) -> Observation:
        t = self.task
        work = tempfile.mkdtemp(prefix="kore_env_")
        try:
            kpath = os.path.join(work, "kernel.py")
            with open(kpath, "w") as f:
                f.write(source)
            os.chmod(kpath, 0o444)
            thr = t.snr_threshold if t.snr_threshold is not None else self.cfg.snr_threshold_for(t.dtype)
            snr_by: Dict[str, float] = {}
            allclose_all = True
            text_tail = ""
            for sh in t.shapes:
                rc, out, to = self._exec(["--task", t.task_id, "--kernel", kpath, "--shape", sh.name,
                                          "--adversarial"], work)
                kind = self._classify(rc, out, to)
                if kind == "infra":
                    return Observation(compiled=True, infra_error=True, error_text=out[-2000:], dtype=t.dtype)
                if kind == "compile":
                    return Observation(compiled=False, error_text=out[-2000:], dtype=t.dtype)
                snrs = _SNR.findall(out)
                acs = _ALLCLOSE.findall(out)
                if not snrs:
                    return Observation(compiled=True, error_text="no verdict: " + out[-1500:], dtype=t.dtype)
                snr_by[sh.name] = float(snrs[-1])
                allclose_all = allclose_all and (acs[-1] == "True" if acs else False)
                text_tail = out[-800:]
            if self.cfg.shape_augment and all(v >= thr for v in snr_by.values()):
                # augmented shapes: correctness only (row-like dims scaled and made non-aligned)
                import json as _json

                from ..tasks.augment import augment_shapes
                for ash in augment_shapes(t, self.cfg.shape_augment_max):
                    rc, out, to = self._exec(["--task", t.task_id, "--kernel", kpath, "--shape", "primary",
                                              "--dims", _json.dumps(ash.dims), "--adversarial"], work)
                    if self._classify(rc, out, to) == "infra":
                        return Observation(compiled=True, infra_error=True, error_text=out[-2000:], dtype=t.dtype)
                    snrs = _SNR.findall(out)
                    snr_by[ash.name] = float(snrs[-1]) if snrs else -999.0
                    if not snrs or float(snrs[-1]) < thr:
                        text_tail = f"fails on augmented shape {ash.as_args()}: " + out[-600:]
                        break
            passed = all(v >= thr for v in snr_by.values())
            obs = Observation(compiled=True, snr_by_shape=snr_by, snr_db=min(snr_by.values()),
                              validation_passed=passed, dtype=t.dtype,
                              error_text=None if passed else text_tail)
            if not passed:
                return obs
            if self.cfg.verifier_determinism_check and not self._deterministic(kpath, work, snr_by, thr):
                obs.validation_passed = False
                obs.error_text = "non-deterministic output (SNR unstable across identical runs)"
                return obs
            self._bench(obs, kpath, work, thr)
            if self.collect_pmc and obs.validation_passed:
                from ..reward.profile_reward import profile_efficiency_score
                from ..verifier.pmc import collect_counters
                obs.counters = collect_counters(self, kpath, work)
                ref = collect_counters(self, kpath, work, impl="baseline") if obs.counters else {}
                if ref:
                    obs.profile_efficiency = profile_efficiency_score(obs.counters, ref)
            return obs
        finally:
            shutil.rmtree(work, ignore_errors=True)

    def _classify(self, rc: int, out: str, timed_out: bool) -> str:
        if timed_out or rc in (-9, -11, 137, 139):
            return "infra"
        if "COMPILE_ERROR" in out:
            return "compile"
        if _INFRA.search(out) and "CANDIDATE_ERROR" not in out:
            return "infra"
        if rc != 0:
            return "compile"
        return "ok"

    def _deterministic(self, kpath, work, snr_by, thr) -> bool:
        prim = self.task.shape("primary") or self.task.shapes[0]
        rc, out, to = self._exec(["--task", self.task.task_id, "--kernel", kpath, "--shape", prim.name], work)
        snrs = _SNR.findall(out)
        if to or not snrs:
            return False
        s2 = float(snrs[-1])
        return s2 >= thr and abs(s2 - snr_by.get(prim.name, s2)) <= self.cfg.determinism_snr_tol_db

    def _bench(self, obs: Observation, kpath, work, thr) -> None:
        shapes = [s.name for s in self.task.bench_shapes()] or [self.task.shapes[0].name]
        cands: Dict[str, List[float]] = {s: [] for s in shapes}
        refs: Dict[str, List[float]] = {s: [] for s in shapes}
        cvs: List[float] = []
        with self._timing_lock():
            for run in range(self.cfg.max_variance_runs):
                rc, out, to = self._exec(["--task", self.task.task_id, "--kernel", kpath, "--bench-both",
                                          "--shapes", ",".join(shapes), "--warmup", str(self.cfg.warmup_iters),
                                          "--iters", str(self.cfg.bench_iters)], work,
                                         timeout=self.timeout * 2)
                if to or rc != 0:
                    obs.error_text = "bench failed: " + (out or "")[-1000:]
                    return
                for kind, name, ms, cv in _BENCH.findall(out):
                    (cands if kind == "CAND" else refs)[name].append(float(ms))
                    if kind == "CAND":
                        cvs.append(float(cv))
                for name, snr in _POST.findall(out):
                    if float(snr) < thr:   # result changed after timing: poisoned / do-less-work
                        obs.validation_passed = False
                        obs.flagged_hack = True
                        obs.hack_reason = f"output changed after timing on {name} (SNR {snr} dB)"
                        return
                if run + 1 >= self.cfg.min_variance_runs and (not cvs or median(cvs) <= self.cfg.cv_threshold_pct):
                    break
        obs.wall_by_shape = {k: median(v) for k, v in cands.items() if v}
        obs.baseline_by_shape = {k: median(v) for k, v in refs.items() if v}
        prim = "primary" if "primary" in obs.wall_by_shape else next(iter(obs.wall_by_shape), None)
        if prim:
            obs.wall_ms = obs.wall_by_shape[prim]
            obs.baseline_ms = obs.baseline_by_shape.get(prim)
        obs.cv_pct = median(cvs) if cvs else None


class KernelRolloutEnv(RolloutEnv):
    """GRPO adapter: prompts from the task, each turn's response parsed for a
    FULL_KERNEL, verified with :class:`KoreEnv`, scored with the kernel reward
    (speedup or residual mode, curriculum phase, roofline gate)."""

    def __init__(self, config, gpu: Optional[int] = None, cache_path: Optional[str] = None):
        self.cfg = config
        self.gpu = gpu
        self.cache = ReplayCache(cache_path) if cache_path else ReplayCache()
        self._envs: Dict[str, KoreEnv] = {}

    def _env(self, task_id: str) -> KoreEnv:
        if task_id not in self._envs:
            self._envs[task_id] = KoreEnv(task_id, gpu=self.gpu, cache=self.cache)
        return self._envs[task_id]

    def prompt_messages(self, task):
        from ..policy.format import SYSTEM_PROMPT, build_task_prompt
        t = get_task(task) if isinstance(task, str) else task
        return [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": build_task_prompt(t)}]

    def step(self, task, response: str, turn: int, traj: int, history) -> TurnResult:
        from ..policy.format import build_turn_feedback, parse_response
        from ..reward.physics import compute_kernel_reward
        from ..reward.whitebox import phi_potential
        env = self._env(task)
        code = parse_response(response).get("kernel", "")
        if not code.strip():
            obs = Observation(compiled=False, error_text="no FULL_KERNEL in response", dtype=env.task.dtype)
        else:
            obs = env.step(code)
        rr = compute_kernel_reward(obs, code, env.task, mode=self.cfg.reward_mode, dtype=env.task.dtype,
                                   response=response, reward_phase=self.cfg.reward_phase,
                                   roofline_gate=self.cfg.roofline_gate, roofline_tol=self.cfg.roofline_tol,
                                   physics_weight=self.cfg.physics_weight)
        return TurnResult(reward=rr.reward, correct=rr.correct, feedback=build_turn_feedback(obs),
                          phi=phi_potential(env.task, obs) if rr.correct else None, infra=obs.infra_error,
                          obs=obs, code=code)
