"""Verifier driver: runs a candidate kernel module for one task in its own
process (the KoreEnv launches it under a timeout, in a new session).

    python -m kore_b200.tasks.driver --task ID --kernel kernel.py --shape primary
    python -m kore_b200.tasks.driver --task ID --kernel kernel.py --bench-both --shapes primary,validation0

Correctness (default): >= 5 reseeded trials plus adversarial fills (zeros,
large magnitudes, tiny values, near-ties, sparse spikes) against the fp32
oracle (a fresh output tensor per call); prints
``SNR: <dB>``, ``allclose: <bool>``, ``max_diff: <x>`` (worst over trials).
Bench (``--bench-both``): for each shape, candidate and vendor baseline are
timed alternately with CUDA events around each call after a 512 MiB L2
flush, with a randomised number of warm-up and timed iterations; prints
``CAND <shape> <median_ms> <cv%>`` / ``REF <shape> <median_ms> <cv%>`` and
re-verifies the candidate's output after timing (``POST_VERIFY_SNR``).
Reference parity: kore/tasks/_genops.py:787-1093 and the per-task driver
contract (tasks/rmsnorm_aiter/driver.py:66-157).
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import os
import random
import sys

import torch

from .ops_library import SPECS
from .registry import get_task

_FLUSH = None


def l2_flush():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def snr_db(out, ref) -> float:
    o, r = out.float(), ref.float()
    finite = torch.isfinite(r)
    if not torch.equal(torch.isfinite(o) | ~finite, torch.ones_like(finite)):
        return -999.0
    o, r = torch.where(finite, o, 0), torch.where(finite, r, 0)
    noise = (o - r).norm().item()
    sig = r.norm().item()
    if noise == 0:
        return 999.0
    return 20 * math.log10(sig / noise) if sig > 0 else -999.0


def task_torch_dtype(dtype: str):
    """Input dtype of a task (fp8 tasks take bf16 inputs and quantise inside)."""
    return {"fp16": torch.float16, "fp32": torch.float32}.get(dtype, torch.bfloat16)


def load_candidate(path: str, entry: str):
    spec = importlib.util.spec_from_file_location("candidate_kernel", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return getattr(mod, entry)


def adversarial(inputs, kind: int):
    """Deterministic hard regimes applied to the floating inputs."""
    out = []
    for t in inputs:
        if not t.is_floating_point():
            out.append(t)
            continue
        x = t.clone()
        if kind == 0:
            x.zero_()
        elif kind == 1:
            x.mul_(100.0)
        elif kind == 2:
            x.mul_(1e-3)
        elif kind == 3:   # near ties
            x.copy_((x.float() * 0.01 + 1.0).to(x.dtype))
        elif kind == 4:   # sparse spikes
            m = torch.rand(x.shape, device=x.device) < 0.001
            x.masked_fill_(m, 50.0)
        out.append(x)
    return tuple(out)


def run_correctness(task, fn, dims, trials: int, atol: float, rtol: float, adv: bool) -> float:
    spec = SPECS[task.spec]
    dt = task_torch_dtype(task.dtype)
    worst, maxd, ok = 999.0, 0.0, True
    cases = [(s, None) for s in range(trials)] + ([(100 + k, k) for k in range(5)] if adv else [])
    for seed, kind in cases:
        inputs = spec.make_inputs(dims, seed, "cuda", dt)
        if kind is not None:
            inputs = adversarial(inputs, kind)
        ref = spec.reference(*inputs)
        try:
            out = fn(*inputs)
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001 - candidate errors are results, not crashes
            print(f"CANDIDATE_ERROR: {type(e).__name__}: {e}")
            print("SNR: -999.00 dB\nallclose: False\nmax_diff: inf")
            return -999.0
        if tuple(out.shape) != tuple(ref.shape):
            print(f"CANDIDATE_ERROR: shape {tuple(out.shape)} != {tuple(ref.shape)}")
            print("SNR: -999.00 dB\nallclose: False\nmax_diff: inf")
            return -999.0
        s = snr_db(out, ref)
        worst = min(worst, s)
        maxd = max(maxd, (out.float() - ref.float()).abs().nan_to_num(float("inf")).max().item())
        ok = ok and torch.allclose(out.float(), ref.float(), atol=atol, rtol=rtol)
    print(f"SNR: {worst:.2f} dB\nallclose: {ok}\nmax_diff: {maxd:.6f}")
    return worst


def time_events(fn, warmup: int, iters: int):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        l2_flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    med = times[len(times) // 2]
    mean = sum(times) / len(times)
    cv = 100.0 * math.sqrt(sum((t - mean) ** 2 for t in times) / len(times)) / mean if mean > 0 else 0.0
    return med, cv


def run_bench(task, fn, shapes, warmup, iters):
    spec = SPECS[task.spec]
    dt = task_torch_dtype(task.dtype)
    rng = random.Random()
    for name in shapes:
        sh = task.shape(name)
        inputs = spec.make_inputs(sh.dims, 0, "cuda", dt)
        w = warmup + rng.randrange(0, 5)
        n = iters + rng.randrange(0, 5)
        # alternate candidate / reference to share clock and thermal state
        cm, ccv = time_events(lambda: fn(*inputs), w, n)
        rm, rcv = time_events(lambda: spec.baseline(*inputs), w, n)
        print(f"CAND {name} {cm:.5f} {ccv:.2f}")
        print(f"REF {name} {rm:.5f} {rcv:.2f}")
        out = fn(*inputs)
        torch.cuda.synchronize()
        print(f"POST_VERIFY_SNR {name} {snr_db(out, spec.reference(*inputs)):.2f}")


def run_profile(task, fn, dims, warmup: int = 2):
    """Warm-up calls, then one call inside the NVTX range ``kore_profile``
    that a counter capture selects (``ncu --nvtx --nvtx-include kore_profile/``)."""
    spec = SPECS[task.spec]
    inputs = spec.make_inputs(dims, 0, "cuda", task_torch_dtype(task.dtype))
    for _ in range(warmup):
        fn(*inputs)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("kore_profile")
    fn(*inputs)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print("PROFILE_RUN_OK")


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--task", required=True)
    p.add_argument("--kernel", required=True)
    p.add_argument("--shape", default="primary")
    p.add_argument("--bench-both", action="store_true")
    p.add_argument("--shapes", default="primary")
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--iters", type=int, default=30)
    p.add_argument("--trials", type=int, default=int(os.environ.get("KORE_CORRECTNESS_TRIALS", "5")))
    p.add_argument("--adversarial", action="store_true")
    p.add_argument("--atol", type=float, default=1e-2)
    p.add_argument("--rtol", type=float, default=1e-2)
    p.add_argument("--dims", default=None, help="JSON dims overriding the named shape's (augmented shapes)")
    p.add_argument("--profile-run", choices=["candidate", "baseline"], default=None,
                   help="run one call of the candidate or the vendor baseline inside an NVTX range "
                        "named kore_profile (for a counter capture), no verification")
    a = p.parse_args(argv)
    task = get_task(a.task)
    try:
        fn = load_candidate(a.kernel, task.entry)
    except Exception as e:  # noqa: BLE001 - import / compile failure of the candidate
        print(f"COMPILE_ERROR: {type(e).__name__}: {e}")
        return 3
    if a.bench_both:
        run_bench(task, fn, [s for s in a.shapes.split(",") if s], a.warmup, a.iters)
        return 0
    if a.profile_run:
        sh = task.shape(a.shape)
        if sh is None:
            print(f"unknown shape {a.shape}", file=sys.stderr)
            return 2
        run_profile(task, fn if a.profile_run == "candidate" else SPECS[task.spec].baseline, sh.dims)
        return 0
    sh = task.shape(a.shape)
    if a.dims:
        import json
        dims = json.loads(a.dims)
    elif sh is None:
        print(f"unknown shape {a.shape}", file=sys.stderr)
        return 2
    else:
        dims = sh.dims
    run_correctness(task, fn, dims, max(5, a.trials), a.atol, a.rtol, a.adversarial)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
