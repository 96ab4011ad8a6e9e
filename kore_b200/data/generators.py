"""Data-factory generators beyond repair / groups / wins / evolve.

* ``gen_qa``: grounded question/answer pairs about kernels and the B200 whose
  answers are computed, not written by a teacher: roofline time and bound of an
  operation at a shape (from the measured-peak roofline model), compulsory
  bytes, arithmetic intensity, which of two verified kernels is faster (from
  measured wins), what class of bug a mutated kernel has (from the mutation
  engine), and hardware facts of the target. Reference: kore/data/gen_qa.py:120-212.
* ``synthetic_inductor_corpus``: kernels written by PyTorch's own compiler for
  the task library's operators, as a continued-pretraining corpus of
  compiler-grade code with the source operator as context.
  Reference: kore/data/synthetic.py:223.
* ``gold_wins``: wins re-verified and re-timed (robust, worst-of-trials) that
  still beat the baseline, deduplicated per task. Reference: kore/data/gold_wins.py:157.
* ``grounded_reasoning``: ANALYSIS / PROPOSED_CHANGE / FULL_KERNEL responses for
  measured (before, after) kernel pairs, with the analysis stating the measured
  numbers (time, roofline fraction, bound, speedup) instead of free text.
  Reference: kore/data/grounded_reasoning.py.
* ``synth_agentic``: tool-use trajectories (build -> test -> bench -> keep) whose
  tool results are the environment's real observations of a win's kernels.
  Reference: kore/data/synth_agentic.py:415.
* ``onpolicy_pairs`` / ``dagger``: the iterative-DPO round: sample the current
  policy on tasks, verify, and pair the best correct response against worse or
  incorrect ones; DAgger relabels the policy's failures with a teacher's
  verified fix. Reference: kore/data/onpolicy.py:96.
"""
from __future__ import annotations

import hashlib
import json
import random
from typing import Callable, Dict, Iterable, List, Optional, Sequence

from .schemas import WinRecord

# B200 facts used by the hardware questions (nominal; measured peaks come from the roofline model)
B200_FACTS = {
    "streaming multiprocessors": "148",
    "warp size (threads)": "32",
    "maximum shared memory per thread block (KB)": "227",
    "tensor memory per SM (KB)": "256",
    "L2 cache (MB)": "126",
    "HBM3e capacity (GB)": "180",
    "NVLink 5 bandwidth per direction per GPU (GB/s)": "900",
    "dense bf16 tensor-core peak (PFLOP/s)": "2.25",
}


def _msgs(q: str, a: str) -> Dict:
    return {"messages": [{"role": "user", "content": q}, {"role": "assistant", "content": a}], "type": "qa"}


# ----------------------------------------------------------------------------- QA
def gen_qa(tasks, *, wins: Iterable[WinRecord] = (), per_task: int = 3, seed: int = 0) -> List[Dict]:
    from ..analysis.rooflines import detect_arch, flops_bytes, resolve_peaks, roofline, shape_to_str
    from .factory import mutate
    rng = random.Random(seed)
    arch = detect_arch()
    peaks = resolve_peaks(arch, use_measured=True)
    out: List[Dict] = []
    for t in tasks:
        prim = t.shape("primary") if hasattr(t, "shape") else None
        dims = getattr(prim, "dims", None) or {}
        fams = []
        fb = flops_bytes(t.operation, dims, t.dtype) if dims else None
        if fb:
            rf = roofline(t.task_id, t.operation, t.dtype, shape_to_str(dims), dims, peaks, arch)
            fams.append(_msgs(f"For {t.operation} ({t.dtype}) at {shape_to_str(dims)} on B200, what is the "
                              f"roofline lower bound on runtime and is it compute- or memory-bound?",
                              f"{rf.t_min_ms:.4g} ms, {rf.bound}-bound (FLOPs {fb[0]:.3g}, compulsory bytes "
                              f"{fb[1]:.3g})."))
            fams.append(_msgs(f"What is the arithmetic intensity (FLOP/byte) of {t.operation} at "
                              f"{shape_to_str(dims)} in {t.dtype}?", f"{fb[0] / max(fb[1], 1.0):.3g} FLOP/byte."))
            fams.append(_msgs(f"How many bytes must {t.operation} at {shape_to_str(dims)} ({t.dtype}) move to "
                              f"and from HBM at minimum?", f"{fb[1]:.4g} bytes."))
        if getattr(t, "seed_src", ""):
            bad, kind = mutate(t.seed_src, rng)
            if bad and bad != t.seed_src:
                fams.append(_msgs("This kernel was changed from a correct version. What kind of bug was "
                                  f"introduced?\n```python\n{bad}\n```", f"A {kind} bug."))
        rng.shuffle(fams)
        out += fams[:per_task]
    wl = [w for w in wins if w.speedup and w.final_kernel]
    for a, b in zip(wl[0::2], wl[1::2]):
        if a.task_id == b.task_id and abs((a.speedup or 0) - (b.speedup or 0)) > 0.05:
            fast, slow = (a, b) if a.speedup > b.speedup else (b, a)
            out.append(_msgs(f"Two verified kernels for {a.task_id}. Which is faster?\n"
                             f"A:\n```python\n{fast.final_kernel}\n```\nB:\n```python\n{slow.final_kernel}\n```",
                             f"A ({fast.speedup:.2f}x vs {slow.speedup:.2f}x over the baseline)."))
    for k, v in B200_FACTS.items():
        out.append(_msgs(f"On an NVIDIA B200, what is the {k}?", v))
    return out


# ----------------------------------------------------------------------------- compiler corpus
def synthetic_inductor_corpus(specs: Sequence, device: str = "cpu", limit: int = 32) -> List[Dict]:
    """Compile each operator's fp32 oracle with torch.compile on ``device`` and
    keep the generated kernel code (one text record per operator)."""
    import torch
    from torch._inductor.utils import run_and_get_code
    out: List[Dict] = []
    for spec in list(specs)[:limit]:
        try:
            x = spec.make_inputs(spec.shapes["minimal"], 0, device, torch.float32)
            fn = torch.compile(lambda *a, f=spec.reference: f(*a), dynamic=False)
            _, codes = run_and_get_code(fn, *x)
        except Exception:  # noqa: BLE001 - operators the compiler rejects are skipped
            continue
        if codes:
            out.append({"text": f"# operator: {spec.name} ({spec.operation})\n# reference:\n"
                                + "\n".join("# " + l for l in spec.seed_src.splitlines()) + "\n\n" + codes[0],
                        "type": "inductor", "task_id": spec.name})
    return out


# ----------------------------------------------------------------------------- gold wins
def gold_wins(wins: Iterable[WinRecord], tasks_by_id: Dict, env_factory, *, min_speedup: float = 1.05,
              trials: int = 2) -> List[WinRecord]:
    from ..eval.suite import robust_eval
    best: Dict[str, WinRecord] = {}
    for w in wins:
        if w.final_kernel and w.task_id in tasks_by_id and (w.task_id not in best or
                                                             (w.speedup or 0) > (best[w.task_id].speedup or 0)):
            best[w.task_id] = w
    out = []
    for tid, w in sorted(best.items()):
        r = robust_eval(tasks_by_id[tid], w.final_kernel, env_factory, trials)
        if r["correct"] and r["speedup"] >= min_speedup:
            w.speedup = r["speedup"]
            out.append(w)
    return out


# ----------------------------------------------------------------------------- grounded reasoning
def grounded_reasoning(task, before: str, after: str, env) -> Optional[Dict]:
    """One SFT record whose analysis quotes the measured numbers of the pair."""
    from ..policy.format import build_task_prompt
    from ..reward.physics import KernelScorer
    ob, oa = env.step(before), env.step(after)
    if not (oa.validation_passed and oa.wall_ms and ob.wall_ms):
        return None
    ev = KernelScorer().evidence(task, oa)
    eb = KernelScorer().evidence(task, ob)
    fa = ev.attainment()[0] if ev else None
    fb = eb.attainment()[0] if eb else None
    lines = [f"The current kernel takes {ob.wall_ms:.4g} ms"
             + (f" ({fb:.0%} of the roofline)" if fb is not None else "") + ".",
             f"The change below runs in {oa.wall_ms:.4g} ms"
             + (f" ({fa:.0%} of the roofline)" if fa is not None else "")
             + f", {ob.wall_ms / oa.wall_ms:.2f}x faster, and stays correct on every shape."]
    if oa.baseline_ms:
        lines.append(f"The vendor baseline takes {oa.baseline_ms:.4g} ms.")
    resp = ("ANALYSIS:\n" + " ".join(lines) + "\n\nPROPOSED_CHANGE:\nApply the rewrite below.\n\n"
            f"FULL_KERNEL:\n```python\n{after}\n```")
    prompt = build_task_prompt(task) + f"\n\nCurrent kernel:\n```python\n{before}\n```"
    return {"messages": [{"role": "user", "content": prompt}, {"role": "assistant", "content": resp}],
            "type": "grounded_reasoning", "task_id": task.task_id,
            "speedup": ob.wall_ms / oa.wall_ms}


# ----------------------------------------------------------------------------- synthetic agentic
def synth_agentic(task, kernels: Sequence[str], env) -> Dict:
    """A Hermes tool-call transcript over ``kernels`` (each built, tested and
    benched; the best verified one kept) with the environment's real results."""
    from ..agent.format import build_agent_system_prompt, format_tool_result
    from ..agent.tools import ToolExecutor
    from ..policy.format import build_task_prompt
    ex = ToolExecutor(env, task, current=getattr(task, "seed_src", ""))
    msgs = [{"role": "system", "content": build_agent_system_prompt(ex.tools())},
            {"role": "user", "content": build_task_prompt(task)}]
    for src in kernels:
        for tool in ("build", "test", "bench"):
            call = {"name": tool, "arguments": {"source": src}}
            msgs.append({"role": "assistant", "content": "<tool_call>\n" + json.dumps(call) + "\n</tool_call>"})
            res = ex.call(tool, call["arguments"])
            msgs.append({"role": "tool", "content": format_tool_result(tool, res)})
            if tool != "bench" and not res.get("correct", res.get("compiled", False)):
                break
    if ex.best:
        msgs.append({"role": "assistant", "content": "<tool_call>\n" + json.dumps(
            {"name": "keep", "arguments": {"source": ex.best}}) + "\n</tool_call>"})
        msgs.append({"role": "tool", "content": format_tool_result("keep", ex.call("keep", {"source": ex.best}))})
    return {"messages": msgs, "type": "synth_agentic", "task_id": task.task_id, "final_kernel": ex.best,
            "best_ms": ex.best_ms}


# ----------------------------------------------------------------------------- on-policy DPO / DAgger
def onpolicy_pairs(tasks, policy: Callable[[object], List[str]], env_factory, *, margin: float = 1.02) -> List[Dict]:
    """``policy(task) -> responses``; each verified, scored with the reward
    ladder; the best response is paired against every clearly worse one."""
    from ..policy.format import build_task_prompt, parse_response
    from ..reward.reward import compute_reward
    out = []
    for t in tasks:
        env = env_factory(t)
        scored = []
        for resp in policy(t):
            code = parse_response(resp).get("kernel", "")
            from ..reward.reward import Observation
            obs = env.step(code) if code.strip() else Observation(compiled=False, error_text="no kernel")
            scored.append((compute_reward(obs, code, dtype=t.dtype).reward, resp))
        scored.sort(key=lambda x: -x[0])
        if len(scored) < 2:
            continue
        best_r, best = scored[0]
        prompt = [{"role": "user", "content": build_task_prompt(t)}]
        for r, resp in scored[1:]:
            if best_r > r * margin + 1e-6 or (best_r > 0 >= r):
                out.append({"prompt": prompt, "chosen": best, "rejected": resp, "task_id": t.task_id,
                            "margin": best_r - r, "type": "onpolicy_dpo"})
    return out


def dagger(tasks, policy: Callable[[object], List[str]], teacher, env_factory, *, margin: float = 1.02) -> List[Dict]:
    """Relabel the policy's failures with the teacher's verified fix."""
    from .curation import dagger_relabel
    return dagger_relabel(tasks, policy, teacher, env_factory, margin=margin)


def dedup(records: Iterable[Dict], key: Callable[[Dict], str]) -> List[Dict]:
    seen, out = set(), []
    for r in records:
        h = hashlib.sha256(key(r).encode()).hexdigest()
        if h not in seen:
            seen.add(h)
            out.append(r)
    return out
