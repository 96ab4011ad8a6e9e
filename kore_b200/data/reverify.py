"""Re-verify and re-baseline stored datagen records under the current verifier.

Records written earlier (by an older verifier, a weaker baseline, fewer
correctness trials or another GPU) are measured again, without the teacher:

* ranked groups: every candidate is evaluated afresh, the group is re-ranked
  by (correct first, then wall time) and its preference pairs are rebuilt with
  a noise margin; a group left without a pair is dropped;
* wins: the final kernel and the task's seed are evaluated afresh; the win is
  dropped when the kernel is no longer correct or no longer beats the seed by
  ``min_speedup``, else its wall times and speedup are updated;
* repairs: the repaired kernel (the last assistant turn's) is verified again
  and the record dropped when it no longer passes.

Measurements are fresh: the environments are built without the replay cache
(a cached observation would turn the re-measure into a no-op), and
``rigorous_env`` raises the driver's correctness trials. Output records are
appended one by one and the keys of handled input records are kept beside
the output, so a re-run skips them and a long re-verification resumes after
an interruption.

    python -m kore_b200.data.reverify --kind groups --inputs old.jsonl --out new.jsonl

Reference parity: kore/data/reverify.py and verify_rigor.py (re-verify,
re-rank, drop stale wins / repairs, resumable), for this repository's
records and verifier.
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import json
import math
import os
from pathlib import Path
from typing import Callable, Dict, Iterator, List, Optional, Tuple

from .schemas import RankedGroupRecord, RepairRecord, WinRecord, read_records, write_records

NOISE_MARGIN = 1.02


@contextlib.contextmanager
def rigorous_env(trials: int = 10) -> Iterator[None]:
    """Raise the driver's correctness trials for everything verified inside."""
    old = os.environ.get("KORE_CORRECTNESS_TRIALS")
    os.environ["KORE_CORRECTNESS_TRIALS"] = str(int(trials))
    try:
        yield
    finally:
        if old is None:
            os.environ.pop("KORE_CORRECTNESS_TRIALS", None)
        else:
            os.environ["KORE_CORRECTNESS_TRIALS"] = old


def record_key(rec) -> str:
    d = rec.to_dict()
    body = json.dumps({k: d.get(k) for k in ("type", "task_id", "parent_id", "parent_hash", "final_kernel")},
                      sort_keys=True)
    if isinstance(rec, RankedGroupRecord):
        body += "".join(c.get("source", "") for c in rec.candidates)
    elif isinstance(rec, RepairRecord):
        body += json.dumps(rec.messages[-1:])
    return hashlib.sha256(body.encode()).hexdigest()[:20]


def _ok(obs) -> bool:
    return bool(obs is not None and obs.compiled and obs.validation_passed and obs.wall_ms)


def rebuild_preferences(cands: List[dict], margin: float = NOISE_MARGIN) -> Tuple[List[int], List[List[int]]]:
    """Rank (correct first, then wall time) and adjacent preference pairs
    whose winner is correct and beats the loser by more than ``margin``."""
    order = sorted(range(len(cands)), key=lambda i: (not cands[i]["correct"], cands[i]["wall_us"] or math.inf))
    prefs = []
    for a, b in zip(order, order[1:]):
        ca, cb = cands[a], cands[b]
        if ca["correct"] and (not cb["correct"] or cb["wall_us"] > margin * ca["wall_us"]):
            prefs.append([a, b])
    return order, prefs


def reverify_group(rec: RankedGroupRecord, env) -> Optional[RankedGroupRecord]:
    parent = env.step(env.task.seed_src)
    cands = []
    for c in rec.candidates:
        obs = env.step(c.get("source", ""))
        ok = _ok(obs)
        nc = dict(c)
        nc.update({"correct": ok, "wall_us": obs.wall_ms * 1e3 if ok else None,
                   "snr_db": obs.snr_db if obs is not None else None})
        cands.append(nc)
    order, prefs = rebuild_preferences(cands)
    if not prefs:
        return None
    for r, i in enumerate(order):
        cands[i]["rank"] = r
    d = rec.to_dict()
    d.update({"candidates": cands, "preferences": prefs,
              "parent_wall_us": parent.wall_ms * 1e3 if _ok(parent) else rec.parent_wall_us})
    return RankedGroupRecord.from_dict(d)


def reverify_win(rec: WinRecord, env, min_speedup: float = 1.0) -> Optional[WinRecord]:
    src = rec.final_kernel or _last_kernel(rec.trajectory)
    if not src:
        return None
    seed, fin = env.step(env.task.seed_src), env.step(src)
    if not (_ok(seed) and _ok(fin)):
        return None
    sp = seed.wall_ms / fin.wall_ms
    if sp <= min_speedup:
        return None
    d = rec.to_dict()
    d.update({"initial_wall_us": seed.wall_ms * 1e3, "final_wall_us": fin.wall_ms * 1e3, "speedup": sp,
              "final_kernel": src})
    return WinRecord.from_dict(d)


def reverify_repair(rec: RepairRecord, env) -> Optional[RepairRecord]:
    src = _last_kernel(rec.messages)
    if not src:
        return None
    obs = env.step(src)
    if not (obs is not None and obs.compiled and obs.validation_passed):
        return None
    d = rec.to_dict()
    d["child_snr_db"] = obs.snr_db
    return RepairRecord.from_dict(d)


def _last_kernel(messages: List[dict]) -> Optional[str]:
    from ..policy.format import parse_response
    for m in reversed(messages or []):
        if m.get("role") == "assistant":
            k = parse_response(m.get("content", ""))["kernel"]
            if k:
                return k
    return None


def reverify_file(inputs: List[str], out_path: str, env_factory: Callable, *, kind: Optional[str] = None,
                  min_speedup: float = 1.0, limit: Optional[int] = None) -> Dict[str, int]:
    """Re-verify every record of ``inputs`` (groups, wins or repairs; ``kind``
    restricts it) into ``out_path``; input records already handled by an
    earlier run (their keys are in ``out_path + ".keys"``) are skipped.
    Returns counts."""
    stats = {"seen": 0, "kept": 0, "dropped": 0, "skipped": 0}
    keys_path = out_path + ".keys"                   # keys of the input records already handled
    done = set(Path(keys_path).read_text().split()) if Path(keys_path).exists() else set()
    envs: Dict[str, object] = {}
    for path in inputs:
        for rec in read_records(path):
            t = {"ranked_group": "groups", "win": "wins", "repair": "repairs"}.get(rec.type, "")
            if kind and t != kind:
                continue
            if limit is not None and stats["seen"] >= limit:
                return stats
            stats["seen"] += 1
            key = record_key(rec)
            if key in done:
                stats["skipped"] += 1
                continue
            env = envs.get(rec.task_id)
            if env is None:
                try:
                    env = envs[rec.task_id] = env_factory(rec.task_id)
                except KeyError:                         # a task this registry does not have
                    stats["dropped"] += 1
                    with open(keys_path, "a") as f:
                        f.write(key + "\n")
                    done.add(key)
                    continue
            if isinstance(rec, RankedGroupRecord):
                new = reverify_group(rec, env)
            elif isinstance(rec, WinRecord):
                new = reverify_win(rec, env, min_speedup)
            else:
                new = reverify_repair(rec, env)
            if new is None:
                stats["dropped"] += 1
            else:
                write_records(out_path, [new])
                stats["kept"] += 1
            with open(keys_path, "a") as f:                # the input record is done, kept or not
                f.write(key + "\n")
            done.add(key)
    return stats


def default_env_factory(gpu: Optional[int] = None):
    from ..env.kore_env import KoreEnv

    def make(task_id: str):
        return KoreEnv(task_id, gpu=gpu, cache=None)
    return make


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore reverify")
    ap.add_argument("--inputs", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--kind", choices=["groups", "wins", "repairs"], default=None)
    ap.add_argument("--trials", type=int, default=10)
    ap.add_argument("--min-speedup", type=float, default=1.0)
    ap.add_argument("--gpu", type=int, default=None)
    ap.add_argument("--limit", type=int, default=None)
    a = ap.parse_args(argv)
    with rigorous_env(a.trials):
        st = reverify_file([p for p in a.inputs.split(",") if p], a.out, default_env_factory(a.gpu),
                           kind=a.kind, min_speedup=a.min_speedup, limit=a.limit)
    print(json.dumps(st))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
