"""Dataset curation beyond the three generators.

* ``hard_negatives``: for each verified kernel, rejected variants that still
  compile but are wrong in instructive ways (dropped mask, wrong reduction,
  fp16 accumulation, off-by-one grid, ...), paired with the correct kernel as
  DPO (chosen, rejected) pairs.
* ``repair_to_dpo``: a repair record becomes a preference pair (repaired
  kernel preferred over the broken parent) on the same prompt.
* ``mix``: multi-capability SFT mixing with per-source weights (sampling with
  replacement to the target size, deterministic under a seed).
* ``midtrain_corpus``: ``{"text"}`` documents from task statements, reference
  oracles and winning kernels (continued pre-training on the domain).
* ``dagger_relabel``: on-policy DAgger / iterative DPO round: the current
  policy answers, a teacher relabels, and (policy, teacher) outputs become
  preference pairs when the verifier ranks the teacher's higher.
* ``general_replay``: rows of a general-capability JSONL mixed into SFT to
  limit forgetting.
* ``parallel_datagen``: one worker process per GPU (``CUDA_VISIBLE_DEVICES``
  pinned), tasks partitioned longest-first, each worker appending to its own
  shard so an interrupted run resumes by skipping finished task ids.
Reference parity: kore/data/hard_negatives.py:374-448, mixing.py:213,
midtrain_corpus.py:475, onpolicy.py:96, general_replay.py:354,
parallel_datagen.py:1-247, build_datasets.py (repair -> DPO).
"""
from __future__ import annotations

import json
import os
import random
import subprocess
import sys
from pathlib import Path
from typing import Callable, Dict, Iterable, List, Optional, Sequence

from .factory import BREAKERS, mutate
from .schemas import RepairRecord, WinRecord


def _prompt(task) -> List[dict]:
    from ..policy.format import SYSTEM_PROMPT, build_task_prompt
    return [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": build_task_prompt(task)}]


def _answer(src: str) -> str:
    from ..policy.format import format_assistant_turn
    return format_assistant_turn("verified kernel", "see code", src)


def hard_negatives(task, good_src: str, env, *, per_kernel: int = 3, seed: int = 0) -> List[dict]:
    """DPO pairs (chosen = verified kernel, rejected = a compiling but wrong mutant)."""
    rng = random.Random(seed)
    out = []
    tried = set()
    for _ in range(4 * per_kernel):
        if len(out) >= per_kernel:
            break
        bad, op = mutate(good_src, rng)
        if bad is None or op in tried:
            continue
        tried.add(op)
        obs = env.step(bad)
        if obs.compiled and not obs.validation_passed:        # wrong, not merely broken
            out.append({"prompt": _prompt(task), "chosen": _answer(good_src), "rejected": _answer(bad),
                        "task_id": task.task_id, "negative": op})
    return out


def repair_to_dpo(records: Iterable[RepairRecord]) -> List[dict]:
    rows = []
    for r in records:
        msgs = list(r.messages)
        if not msgs or msgs[-1]["role"] != "assistant":
            continue
        prompt = msgs[:-1]
        broken = next((m["content"] for m in prompt if m["role"] == "user"), "")
        rows.append({"prompt": prompt, "chosen": msgs[-1]["content"],
                     "rejected": "The kernel is correct as written.\n" + broken[-4000:], "task_id": r.task_id})
    return rows


def mix(sources: Dict[str, List[dict]], weights: Dict[str, float], total: int, seed: int = 0) -> List[dict]:
    rng = random.Random(seed)
    names = [n for n in sources if sources[n] and weights.get(n, 0) > 0]
    wsum = sum(weights[n] for n in names)
    out = []
    for n in names:
        k = int(round(total * weights[n] / wsum))
        pool = sources[n]
        out += [dict(pool[rng.randrange(len(pool))], source=n) for _ in range(k)]
    rng.shuffle(out)
    return out[:total]


def midtrain_corpus(tasks, wins: Iterable[WinRecord] = (), out_path: Optional[str] = None) -> List[dict]:
    docs = []
    for t in tasks:
        docs.append({"text": f"# Task {t.task_id} ({t.operation}, {t.dtype})\n\nShapes: {t.shapes_text}\n\n"
                             f"Reference:\n```python\n{t.reference_src}\n```\n\nSeed kernel:\n```python\n"
                             f"{t.seed_src}\n```\n"})
    for w in wins:
        if w.final_kernel:
            docs.append({"text": f"# Optimised kernel for {w.task_id} ({(w.speedup or 0):.2f}x)\n\n```python\n"
                                 f"{w.final_kernel}\n```\n"})
    if out_path:
        Path(out_path).parent.mkdir(parents=True, exist_ok=True)
        with open(out_path, "w") as f:
            for d in docs:
                f.write(json.dumps(d) + "\n")
    return docs


def dagger_relabel(tasks, policy, teacher, env_factory, *, margin: float = 1.02) -> List[dict]:
    """One on-policy round: pairs where the teacher's kernel verifies and beats
    the policy's (or the policy's fails)."""
    from ..policy.format import parse_response
    pairs = []
    for t in tasks:
        env = env_factory(t)
        msgs = _prompt(t)
        pr, tr = policy.generate(msgs), teacher.generate(msgs)
        po, to = env.step(parse_response(pr)["kernel"] or ""), env.step(parse_response(tr)["kernel"] or "")
        t_ok = to.compiled and to.validation_passed and to.wall_ms
        p_ok = po.compiled and po.validation_passed and po.wall_ms
        if t_ok and (not p_ok or po.wall_ms > margin * to.wall_ms):
            pairs.append({"prompt": msgs, "chosen": tr, "rejected": pr, "task_id": t.task_id})
    return pairs


def general_replay(path: str, n: int, seed: int = 0) -> List[dict]:
    rows = [json.loads(l) for l in open(path) if l.strip()]
    rng = random.Random(seed)
    return [rows[rng.randrange(len(rows))] for _ in range(min(n, len(rows)) if rows else 0)]


def parallel_datagen(kind: str, task_ids: Sequence[str], gpus: Sequence[int], out_dir: str,
                     costs: Optional[Dict[str, float]] = None, extra: Sequence[str] = (),
                     launcher: Callable = subprocess.Popen) -> List[str]:
    """Spawn one ``kore datagen`` worker per GPU over an LPT partition of the
    tasks; skips task ids already present in a worker's shard (resume)."""
    from ..campaign.nodes import lpt_partition
    os.makedirs(out_dir, exist_ok=True)
    done = set()
    for f in Path(out_dir).glob(f"{kind}-gpu*.jsonl"):
        for line in open(f):
            try:
                done.add(json.loads(line).get("task_id"))
            except json.JSONDecodeError:
                continue
    todo = [t for t in task_ids if t not in done]
    parts = lpt_partition({t: (costs or {}).get(t, 1.0) for t in todo}, len(gpus))
    shards, procs = [], []
    for g, part in zip(gpus, parts):
        if not part:
            continue
        shard = os.path.join(out_dir, f"{kind}-gpu{g}.jsonl")
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(g))
        cmd = [sys.executable, "-m", "kore_b200.cli", "datagen", kind, "--tasks", ",".join(part), "--out", shard,
               *extra]
        procs.append(launcher(cmd, env=env))
        shards.append(shard)
    for p in procs:
        if hasattr(p, "wait"):
            p.wait()
    return shards
