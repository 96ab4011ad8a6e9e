"""Data factory: generators that turn teacher proposals into verified records.

* ``generate_repairs``: mutate a correct kernel with a *breaker* (syntax
  slip, wrong mask, wrong constant, dropped normalisation, ...) until the
  verifier rejects it, then ask the teacher to repair it; keep repairs that
  verify (RepairRecord, SFT).
* ``generate_groups``: ask the teacher for k candidate optimisations of a
  parent, verify and time each, rank correct ones by speed; adjacent ranks
  become preference pairs (RankedGroupRecord, DPO).
* ``generate_wins``: multi-turn refinement with verifier feedback; keep
  trajectories whose final kernel beats the initial one (WinRecord).
* ``evolve``: MAP-Elites archive over (tile size bucket, num_warps) with a
  discounted multi-armed bandit over mutation operators (D-MAB).
All generators run against :class:`KoreEnv` on B200, are resumable (they
append JSONL), and accept any teacher. CLI: ``kore datagen {kind} ...``.
Reference parity: kore/data/gen_repair.py:681, gen_groups.py:170,
gen_wins.py:370, evolve.py:352, mutate.py:30-362.
"""
from __future__ import annotations

import argparse
import hashlib
import math
import random
import re
from typing import Callable, Dict, List, Optional, Sequence, Tuple

from ..obs import get_logger
from .knowledge import ExperienceLedger, generation_messages
from ..policy.format import (SYSTEM_PROMPT, build_task_prompt, build_turn_feedback, format_assistant_turn,
                             parse_response)
from .schemas import RankedGroupRecord, RepairRecord, WinRecord, write_records

log = get_logger("data.factory")


# ---------------------------------------------------------------- breakers
def _sub_first(pat, repl):
    def f(src: str) -> Optional[str]:
        out, n = re.subn(pat, repl, src, count=1)
        return out if n else None
    return f


BREAKERS: Dict[str, Callable[[str], Optional[str]]] = {
    "drop_mask": _sub_first(r", mask=m(, other=[^)]*)?\)", ")"),
    "off_by_one_grid": _sub_first(r"\(M,\)", "(M - 1,)"),
    "wrong_eps": _sub_first(r"\+ eps\)", "+ 1.0)"),
    "fp16_accum": _sub_first(r"tl\.float32", "tl.float16"),
    "swap_operands": _sub_first(r"a \* b", "a * a"),
    "syntax_slip": _sub_first(r"\):\n", ")\n"),
    "wrong_reduction": _sub_first(r"tl\.sum\(", "tl.max("),
    "drop_store_cast": _sub_first(r"\.to\(Y\.dtype\.element_ty\)", ".to(tl.float16)"),
    "exp_to_exp2": _sub_first(r"tl\.exp\(", "tl.exp2("),
    "half_block": _sub_first(r"BLOCK=triton\.next_power_of_2\(N\)", "BLOCK=triton.next_power_of_2(N) // 2"),
    "wrong_axis": _sub_first(r"axis=1\)", "axis=0)"),
    "drop_normalization": _sub_first(r"\s*/\s*N\b", ""),
    "transpose_strides": _sub_first(r"stride_am, stride_ak", "stride_ak, stride_am"),
    "drop_scale": _sub_first(r"\s*\*\s*scale\b", ""),
    "fp8_variant": _sub_first(r"float8e4nv", "float8e5"),
    # CUDA C++ sources (inline extensions)
    "drop_syncthreads": _sub_first(r"__syncthreads\(\);", ";"),
    "cuda_bound_off_by_one": _sub_first(r"(if\s*\(\s*\w+\s*)<(\s*\w+\s*\))", r"\1<=\2"),
    "wrong_thread_index": _sub_first(r"threadIdx\.x", "threadIdx.y"),
    "wrong_shuffle_offset": _sub_first(r"(__shfl_xor_sync\([^,]+,[^,]+,\s*)(\w+)", r"\g<1>(\2 + 1)"),
    "cuda_half_accum": _sub_first(r"\bfloat(\s+acc\b)", r"__half\1"),
}

# what each breaker does, for analysis of repair data and the teacher's context
BREAKER_HINTS: Dict[str, str] = {
    "drop_mask": "a bounds mask was removed: the last partial tile reads / writes out of range",
    "off_by_one_grid": "the grid misses the last program: rows at the end stay unwritten",
    "wrong_eps": "the normalisation epsilon is wrong",
    "fp16_accum": "the accumulator is fp16: long reductions lose precision",
    "swap_operands": "an operand was replaced by another",
    "syntax_slip": "a missing colon: the module does not compile",
    "wrong_reduction": "max instead of sum in a reduction",
    "drop_store_cast": "the output is cast to the wrong dtype",
    "exp_to_exp2": "exp2 without the log2(e) scale",
    "half_block": "the block covers half a row: the tail is not processed",
    "wrong_axis": "a reduction runs over the wrong axis",
    "drop_normalization": "the division by N of a mean is missing",
    "transpose_strides": "an operand is read transposed (strides swapped)",
    "drop_scale": "a scale factor (softmax / quantisation) is missing",
    "fp8_variant": "the fp8 encoding is e5m2 instead of e4m3",
    "drop_syncthreads": "a block barrier was removed: shared-memory race",
    "cuda_bound_off_by_one": "a bounds check admits one element too many: out-of-range access",
    "wrong_thread_index": "the y thread index is used instead of x",
    "wrong_shuffle_offset": "a warp-shuffle reduction uses the wrong lane offset",
    "cuda_half_accum": "a CUDA accumulator is fp16: precision loss",
}


def mutate(src: str, rng: random.Random, names: Optional[Sequence[str]] = None) -> Tuple[Optional[str], str]:
    order = list(names or BREAKERS)
    rng.shuffle(order)
    for n in order:
        out = BREAKERS[n](src)
        if out is not None and out != src:
            return out, n
    return None, ""


def src_hash(src: str) -> str:
    return hashlib.sha256(src.encode()).hexdigest()[:16]


def _messages(task, current: str, feedback: Optional[str] = None) -> List[dict]:
    from copy import copy
    t = copy(task)
    t.seed_src = current
    msgs = [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": build_task_prompt(t)}]
    if feedback:
        msgs[-1]["content"] += f"\n\nVerifier feedback on the current kernel:\n{feedback}"
    return msgs


# ---------------------------------------------------------------- generators
def generate_repairs(tasks, teacher, env_factory, *, per_task: int = 2, seed: int = 0,
                     out_path: Optional[str] = None) -> List[RepairRecord]:
    rng = random.Random(seed)
    out = []
    for task in tasks:
        env = env_factory(task)
        for _ in range(per_task):
            broken, op = mutate(task.seed_src, rng)
            if broken is None:
                continue
            obs = env.step(broken)
            if obs.compiled and obs.validation_passed:
                continue                       # the breaker did not break it
            fail = "compile_fail" if not obs.compiled else "snr_fail"
            fb = build_turn_feedback(obs)
            msgs = _messages(task, broken, fb)
            resp = teacher.generate(generation_messages(msgs, task))
            fixed = parse_response(resp)["kernel"]
            if not fixed:
                continue
            child = env.step(fixed)
            if child.compiled and child.validation_passed:
                rec = RepairRecord(task_id=task.task_id, failure_class=fail, parent_hash=src_hash(broken),
                                   error_text=fb[-2000:], messages=msgs + [{"role": "assistant", "content": resp}],
                                   child_snr_db=child.snr_db, operator=op, operation=task.operation)
                out.append(rec)
    if out_path:
        write_records(out_path, out)
    return out


def generate_groups(tasks, teacher, env_factory, *, k: int = 4, out_path: Optional[str] = None
                    ) -> List[RankedGroupRecord]:
    out = []
    for task in tasks:
        env = env_factory(task)
        parent = env.step(task.seed_src)
        cands = []
        ledger = ExperienceLedger()
        for i in range(k):
            resp = teacher.generate(generation_messages(_messages(task, task.seed_src), task, ledger))
            src = parse_response(resp)["kernel"]
            if not src:
                continue
            obs = env.step(src)
            ok = obs.compiled and obs.validation_passed and obs.wall_ms
            ledger.record(task.task_id, task.seed_src, src, compiled=obs.compiled,
                          correct=bool(obs.validation_passed), parent_ms=parent.wall_ms, child_ms=obs.wall_ms,
                          error=obs.error_text or "")
            cands.append({"source": src, "response": resp, "wall_us": (obs.wall_ms or 0) * 1e3 if ok else None,
                          "snr_db": obs.snr_db, "correct": bool(ok)})
        ranked = sorted(range(len(cands)), key=lambda i: (not cands[i]["correct"],
                                                          cands[i]["wall_us"] or math.inf))
        for r, i in enumerate(ranked):
            cands[i]["rank"] = r
        prefs = [[ranked[j], ranked[j + 1]] for j in range(len(ranked) - 1)
                 if cands[ranked[j]]["correct"] and (not cands[ranked[j + 1]]["correct"] or
                                                     cands[ranked[j + 1]]["wall_us"] > 1.02 * cands[ranked[j]]["wall_us"])]
        if prefs:
            out.append(RankedGroupRecord(task_id=task.task_id, parent_id=src_hash(task.seed_src), candidates=cands,
                                         preferences=prefs, operation=task.operation,
                                         parent_wall_us=(parent.wall_ms or 0) * 1e3 or None))
    if out_path:
        write_records(out_path, out)
    return out


def generate_wins(tasks, teacher, env_factory, *, turns: int = 3, min_speedup: float = 1.05,
                  out_path: Optional[str] = None, ledger: Optional[ExperienceLedger] = None) -> List[WinRecord]:
    """Multi-turn optimisation trajectories that end faster than the seed. The
    teacher sees the B200 playbook and the ledger of this task's failed or
    slower attempts (shared across calls when ``ledger`` is passed); the
    stored trajectory keeps the canonical system prompt and feedback only."""
    out = []
    ledger = ledger if ledger is not None else ExperienceLedger()
    for task in tasks:
        env = env_factory(task)
        first = env.step(task.seed_src)
        if not (first.validation_passed and first.wall_ms):
            continue
        cur, best_ms, best_src = task.seed_src, first.wall_ms, task.seed_src
        msgs = _messages(task, cur)
        traj = list(msgs)
        for _ in range(turns):
            resp = teacher.generate(generation_messages(traj, task, ledger))
            traj.append({"role": "assistant", "content": resp})
            src = parse_response(resp)["kernel"]
            obs = env.step(src) if src else None
            traj.append({"role": "user", "content": "Verifier feedback:\n" + build_turn_feedback(obs)})
            if obs is not None:
                ledger.record(task.task_id, cur, src, compiled=obs.compiled, correct=bool(obs.validation_passed),
                              parent_ms=best_ms, child_ms=obs.wall_ms, error=obs.error_text or "")
            if obs is not None and obs.validation_passed and obs.wall_ms and obs.wall_ms < best_ms:
                best_ms, best_src = obs.wall_ms, src
                cur = src
        sp = first.wall_ms / best_ms
        if sp >= min_speedup:
            out.append(WinRecord(task_id=task.task_id, trajectory=traj, initial_wall_us=first.wall_ms * 1e3,
                                 final_wall_us=best_ms * 1e3, speedup=sp, operation=task.operation,
                                 final_kernel=best_src))
    if out_path:
        write_records(out_path, out)
    return out


class DiscountedBandit:
    """D-MAB over mutation operators: discounted mean reward + UCB bonus."""

    def __init__(self, arms: Sequence[str], gamma: float = 0.9, c: float = 0.5, seed: int = 0):
        self.arms = list(arms)
        self.n = {a: 0.0 for a in arms}
        self.s = {a: 0.0 for a in arms}
        self.gamma, self.c = gamma, c
        self.rng = random.Random(seed)

    def pick(self) -> str:
        tot = sum(self.n.values()) + 1
        for a in self.arms:
            if self.n[a] == 0:
                return a
        return max(self.arms, key=lambda a: self.s[a] / self.n[a] + self.c * math.sqrt(math.log(tot) / self.n[a]))

    def update(self, arm: str, r: float) -> None:
        for a in self.arms:
            self.n[a] *= self.gamma
            self.s[a] *= self.gamma
        self.n[arm] += 1
        self.s[arm] += r


def evolve(task, teacher, env, *, iterations: int = 8, seed: int = 0) -> Dict[tuple, dict]:
    """MAP-Elites over (block-size bucket, num_warps); the teacher proposes a
    child of an elite, the bandit chooses which refinement hint to send."""
    hints = ["increase tile size", "decrease tile size", "change num_warps", "vectorize loads",
             "fuse the reduction", "reduce register pressure"]
    bandit = DiscountedBandit(hints, seed=seed)
    archive: Dict[tuple, dict] = {}

    def cell(src):
        b = re.search(r"BLOCK[_A-Z]*\s*=\s*(\d+)", src)
        w = re.search(r"num_warps\s*=\s*(\d+)", src)
        return (int(math.log2(int(b.group(1)))) if b else -1, int(w.group(1)) if w else -1)

    base = env.step(task.seed_src)
    if base.validation_passed and base.wall_ms:
        archive[cell(task.seed_src)] = {"src": task.seed_src, "ms": base.wall_ms}
    rng = random.Random(seed)
    for _ in range(iterations):
        if not archive:
            break
        parent = archive[rng.choice(list(archive))]
        hint = bandit.pick()
        msgs = _messages(task, parent["src"], f"Try to {hint}.")
        src = parse_response(teacher.generate(msgs))["kernel"]
        obs = env.step(src) if src else None
        gain = 0.0
        if obs is not None and obs.validation_passed and obs.wall_ms:
            c = cell(src)
            gain = max(0.0, parent["ms"] / obs.wall_ms - 1.0)
            if c not in archive or obs.wall_ms < archive[c]["ms"]:
                archive[c] = {"src": src, "ms": obs.wall_ms}
        bandit.update(hint, gain)
    return archive


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore datagen")
    ap.add_argument("kind", choices=["repair", "groups", "wins", "evolve", "agentic", "qa"])
    ap.add_argument("--teacher", default="stub")
    ap.add_argument("--teacher-model", default="")
    ap.add_argument("--base-url", default="")
    ap.add_argument("--tasks", default="")
    ap.add_argument("--out", required=False, default="data/datagen.jsonl")
    ap.add_argument("--gpu", type=int, default=None)
    a = ap.parse_args(argv)
    from ..env.kore_env import KoreEnv
    from ..tasks.registry import all_tasks, get_task
    from .teacher import make_teacher
    kw = {}
    if a.teacher in ("vllm", "http", "claude"):
        kw = {"model": a.teacher_model}
        if a.base_url:
            kw["base_url"] = a.base_url
    teacher = make_teacher(a.teacher, resilient=a.teacher != "stub", **kw)
    tasks = [get_task(t) for t in a.tasks.split(",") if t] or all_tasks()
    factory = lambda t: KoreEnv(t, gpu=a.gpu)
    if a.kind == "repair":
        n = len(generate_repairs(tasks, teacher, factory, out_path=a.out))
    elif a.kind == "groups":
        n = len(generate_groups(tasks, teacher, factory, out_path=a.out))
    elif a.kind == "wins":
        n = len(generate_wins(tasks, teacher, factory, out_path=a.out))
    elif a.kind == "evolve":
        n = sum(len(evolve(t, teacher, factory(t))) for t in tasks)
    else:
        from . import agentic_gen
        n = agentic_gen.main(a.kind, tasks, teacher, factory, a.out)
    log.info("datagen done", kind=a.kind, records=n, out=a.out)
    return 0
