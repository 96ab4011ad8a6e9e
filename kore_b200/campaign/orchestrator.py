"""Staged training campaign with a resumable manifest.

Stages, in order: ``reverify, datagen, evolve, agentic, build, midtrain,
sft, dpo, grpo, soup, eval``. Each stage is a callable taking the campaign
context and returning a dict of outputs (paths, metrics); a stage that
finished is recorded in ``<out>/manifest.json`` with its inputs' digest, so a
re-run skips it unless ``--force`` names it or its inputs changed. Training
stages render a resolved JSON config into the campaign directory and launch
``torchrun -m kore_b200.policy.<stage>`` on the chosen GPUs. The GRPO stage
runs a two-phase curriculum (phase 1 rewards correctness only, phase 2 the
latency term). The retention gate after ``soup`` / ``eval`` stops the
campaign when general-capability scores regress beyond epsilon.
Reference parity: scripts/run_campaign.py:73-79 (stages), :394-490
(manifest resume), :181-232 (launch), :620 (split), :697 (free GPUs),
:1639-1657 (GRPO phases), :1861-1952 (retention hard stop).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, List, Optional

from ..obs import get_logger

log = get_logger("campaign")

STAGES = ["reverify", "datagen", "evolve", "agentic", "build", "midtrain", "sft", "dpo", "dpo_iterative", "grpo",
          "soup", "eval"]
OPTIONAL_STAGES = {"dpo_iterative"}     # run only when configured or asked for by name
TRAIN_STAGES = {"midtrain", "sft", "dpo", "grpo"}


@dataclass
class Campaign:
    out_dir: Path
    base_model: str
    gpus: int = 8
    gpu_ids: Optional[List[int]] = None
    configs: Dict[str, dict] = field(default_factory=dict)     # stage -> config overrides
    dry_run: bool = False
    teacher: str = "stub"
    retention_epsilon: float = 0.005
    retention_suites: Dict[str, str] = field(default_factory=dict)

    @property
    def manifest_path(self) -> Path:
        return self.out_dir / "manifest.json"

    def load_manifest(self) -> dict:
        if self.manifest_path.exists():
            try:
                return json.loads(self.manifest_path.read_text())
            except json.JSONDecodeError:
                log.warn("manifest unreadable; starting over", path=str(self.manifest_path))
        return {"stages": {}}

    def save_manifest(self, m: dict) -> None:
        self.out_dir.mkdir(parents=True, exist_ok=True)
        tmp = self.manifest_path.with_suffix(".tmp")
        tmp.write_text(json.dumps(m, indent=2))
        os.replace(tmp, self.manifest_path)            # atomic: a crash never leaves half a manifest


def _digest(obj) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, default=str).encode()).hexdigest()[:16]


# ------------------------------------------------------------------ stage bodies
def _latest_model(c: Campaign, m: dict) -> str:
    for st in ("soup", "grpo", "dpo_iterative", "dpo", "sft", "midtrain"):
        o = m["stages"].get(st, {}).get("outputs", {})
        if o.get("model"):
            return o["model"]
    return c.base_model


def launch_stage(c: Campaign, stage: str, cfg: dict, port: int = 29511) -> int:
    """Render the resolved config and torchrun the stage on the campaign GPUs."""
    d = c.out_dir / stage
    d.mkdir(parents=True, exist_ok=True)
    path = d / "config.json"
    path.write_text(json.dumps(cfg, indent=2))
    from ..cli import launch_command
    cmd = launch_command(stage, str(path), c.gpus, port)
    env = dict(os.environ)
    if c.gpu_ids is not None:
        env["CUDA_VISIBLE_DEVICES"] = ",".join(map(str, c.gpu_ids))
    log.info("launch", stage=stage, cmd=" ".join(cmd))
    if c.dry_run:
        return 0
    return subprocess.call(cmd, env=env)


def _train_stage(stage: str):
    def run(c: Campaign, m: dict) -> dict:
        data = m["stages"].get("build", {}).get("outputs", {})
        cfg = {"model_name_or_path": _latest_model(c, m) if stage != "dpo" else _latest_model(c, m),
               "output_dir": str(c.out_dir / stage / "model")}
        if stage in ("sft", "dpo", "midtrain") and data.get(stage):
            cfg["dataset_path"] = data[stage]
        cfg.update(c.configs.get(stage, {}))
        if stage == "grpo":
            return _grpo_two_phase(c, cfg)
        rc = launch_stage(c, stage, cfg)
        if rc != 0:
            raise RuntimeError(f"stage {stage} exited {rc}")
        return {"model": cfg["output_dir"]}
    return run


def _grpo_two_phase(c: Campaign, cfg: dict) -> dict:
    """Phase 1: correctness-only reward; phase 2: latency term, from phase 1's weights."""
    p1 = dict(cfg, reward_phase="correctness", output_dir=str(c.out_dir / "grpo" / "phase1"))
    p1["num_steps"] = cfg.get("phase1_steps", max(1, cfg.get("num_steps", 100) // 3))
    if launch_stage(c, "grpo", p1) != 0:
        raise RuntimeError("grpo phase 1 failed")
    p2 = dict(cfg, reward_phase="latency", model_name_or_path=p1["output_dir"])
    if launch_stage(c, "grpo", p2, port=29512) != 0:
        raise RuntimeError("grpo phase 2 failed")
    return {"model": p2["output_dir"], "phase1": p1["output_dir"]}


def _stage_reverify(c: Campaign, m: dict) -> dict:
    """Write the train / held-out split; with ``configs["reverify"]["inputs"]``
    (earlier datagen JSONL files) also re-measure those records under the
    current verifier into ``data/reverified.jsonl``."""
    from ..tasks.registry import split_tasks
    tr, ho = split_tasks()
    p = c.out_dir / "split.json"
    p.write_text(json.dumps({"train": tr, "heldout": ho}))
    out = {"split": str(p), "n_train": len(tr), "n_heldout": len(ho)}
    inputs = (c.configs.get("reverify") or {}).get("inputs") or []
    if inputs and not c.dry_run:
        from ..data.reverify import default_env_factory, reverify_file, rigorous_env
        dst = c.out_dir / "data" / "reverified.jsonl"
        dst.parent.mkdir(parents=True, exist_ok=True)
        with rigorous_env((c.configs.get("reverify") or {}).get("trials", 10)):
            out["reverify"] = reverify_file(list(inputs), str(dst), default_env_factory())
        out["reverified"] = str(dst)
    return out


def _datagen(kind: str):
    def run(c: Campaign, m: dict) -> dict:
        from ..data import factory
        out = str(c.out_dir / "data" / f"{kind}.jsonl")
        if not c.dry_run:
            tr = json.loads((c.out_dir / "split.json").read_text())["train"] if (c.out_dir / "split.json").exists() else []
            factory.main([kind, "--teacher", c.teacher, "--out", out] + (["--tasks", ",".join(tr)] if tr else []))
        return {kind: out}
    return run


def _stage_datagen(c: Campaign, m: dict) -> dict:
    out = {}
    for k in ("repair", "groups", "wins"):
        out.update(_datagen(k)(c, m))
    return out


def _stage_build(c: Campaign, m: dict) -> dict:
    from ..data import build_datasets
    d = c.out_dir / "data"
    out = {}
    for kind in ("sft", "dpo"):
        p = str(d / f"{kind}_train.jsonl")
        srcs = [str(q) for q in sorted(d.glob("*.jsonl")) if not q.name.endswith("_train.jsonl")]
        if not c.dry_run and srcs:
            build_datasets.main([kind, "--inputs", ",".join(srcs), "--out", p])
        out[kind] = p
    mp = str(d / "midtrain_corpus.jsonl")
    if not c.dry_run:
        from ..data.midtrain_corpus import build_midtrain_corpus
        from ..data.schemas import WinRecord, read_records
        wins = [w for q in sorted(d.glob("wins*.jsonl")) for w in read_records(str(q), WinRecord)]
        mc = dict(c.configs.get("midtrain_corpus", {}))
        rep = build_midtrain_corpus(mp, wins=wins, **mc)
        out["midtrain_docs"] = rep["docs"]
    out["midtrain"] = mp
    return out


def _stage_dpo_iterative(c: Campaign, m: dict, policy_factory=None, env_factory=None) -> dict:
    """On-policy iterative DPO (+ DAgger): each round samples the current model
    on the training tasks, pairs its best verified response against worse ones,
    and trains a DPO round (IPO + SFT loss) from that model. Reference:
    scripts/run_campaign.py:1425 and kore/data/onpolicy.py:96."""
    cfg = dict(c.configs.get("dpo_iterative", {}))
    rounds = int(cfg.pop("rounds", 2))
    n_tasks = int(cfg.pop("tasks", 64))
    samples = int(cfg.pop("samples_per_task", 4))
    model = _latest_model(c, m)
    history = []
    for r in range(rounds):
        d = c.out_dir / "dpo_iterative" / f"round{r}"
        d.mkdir(parents=True, exist_ok=True)
        pairs_path = d / "pairs.jsonl"
        if not c.dry_run:
            from ..data.generators import onpolicy_pairs
            from ..tasks.registry import get_task, split_tasks
            train, _ = split_tasks()
            tasks = [get_task(t) for t in train[:n_tasks]]
            if policy_factory is None:
                from ..policy.format import SYSTEM_PROMPT, build_task_prompt
                from ..policy.serve import KorePolicy
                pol = KorePolicy(model, temperature=1.0)
                policy_factory = lambda _m: (lambda t: pol.chat(
                    [[{"role": "system", "content": SYSTEM_PROMPT},
                      {"role": "user", "content": build_task_prompt(t)}]] * samples))
            if env_factory is None:
                from ..env.kore_env import KoreEnv
                env_factory = lambda t: KoreEnv(t.task_id)
            pairs = onpolicy_pairs(tasks, policy_factory(model), env_factory)
            with open(pairs_path, "w") as f:
                for p in pairs:
                    f.write(json.dumps(p) + "\n")
        dcfg = {"model_name_or_path": model, "output_dir": str(d / "model"), "dataset_path": str(pairs_path),
                "loss_type": ["ipo", "sft"]}
        dcfg.update(cfg)
        if launch_stage(c, "dpo", dcfg, port=29521 + r) != 0:
            raise RuntimeError(f"iterative DPO round {r} failed")
        model = dcfg["output_dir"]
        history.append(model)
    return {"model": model, "rounds": history}


def _stage_soup(c: Campaign, m: dict) -> dict:
    from ..policy.configs import SoupConfig
    from ..policy.soup import build_soup
    kore = _latest_model(c, m)
    out = str(c.out_dir / "soup")
    if c.dry_run:
        return {"model": out}
    res = build_soup(SoupConfig(base_model_id=c.base_model, kore_checkpoint=kore, output_dir=out))
    return {"model": res.get("output_dir", out), "alpha": res.get("alpha")}


def _stage_eval(c: Campaign, m: dict) -> dict:
    from ..eval import cli as ecli
    out = str(c.out_dir / "eval.json")
    if not c.dry_run:
        ecli.main(["--model", _latest_model(c, m), "--out", out])
    return {"report": out}


STAGE_FNS: Dict[str, Callable[[Campaign, dict], dict]] = {
    "reverify": _stage_reverify, "datagen": _stage_datagen, "evolve": _datagen("evolve"),
    "agentic": _datagen("agentic"), "build": _stage_build, "midtrain": _train_stage("midtrain"),
    "sft": _train_stage("sft"), "dpo": _train_stage("dpo"), "dpo_iterative": _stage_dpo_iterative,
    "grpo": _train_stage("grpo"),
    "soup": _stage_soup, "eval": _stage_eval,
}


class RetentionStop(RuntimeError):
    pass


def retention_check(c: Campaign, m: dict, generate_factory: Optional[Callable[[str], Callable]] = None) -> None:
    """Hard stop when the latest model regresses general capability.

    ``generate_factory(model) -> generate``: with ``retention_suites`` (name ->
    JSONL of {"prompt", "answer"|"tests"}) the generate callable maps a prompt
    string to text; without them the bundled six-benchmark suite
    (kore_b200.eval.retention) is used and generate maps chat messages to text."""
    if generate_factory is None:
        return
    from ..eval.gates import retention_gate
    cache = str(c.out_dir / "retention_cache.json")
    cur_model = _latest_model(c, m)
    if c.retention_suites:
        from ..eval.gates import run_retention_suite
        base = run_retention_suite(generate_factory(c.base_model), c.retention_suites, cache, c.base_model)
        cur = run_retention_suite(generate_factory(cur_model), c.retention_suites, cache, cur_model)
    else:
        from ..eval.retention import run_retention_suite as run_bundled
        base = run_bundled(generate_factory(c.base_model), cache_path=cache, model_key=c.base_model)
        cur = run_bundled(generate_factory(cur_model), cache_path=cache, model_key=cur_model)
    g = retention_gate(base, cur, c.retention_epsilon)
    m["retention"] = {"base": base, "current": cur, "passed": g.passed}
    if not g.passed:
        raise RetentionStop(g.detail)


def run(c: Campaign, stages: Optional[List[str]] = None, force: Optional[List[str]] = None,
        generate_factory=None) -> dict:
    m = c.load_manifest()
    todo = [s for s in STAGES if (stages is None and (s not in OPTIONAL_STAGES or s in c.configs))
            or (stages is not None and s in stages)]
    for st in todo:
        inputs = {"cfg": c.configs.get(st, {}), "base": c.base_model,
                  "upstream": {k: v.get("outputs") for k, v in m["stages"].items() if STAGES.index(k) < STAGES.index(st)}}
        dig = _digest(inputs)
        prev = m["stages"].get(st)
        if prev and prev.get("status") == "done" and prev.get("digest") == dig and st not in (force or []):
            log.info("skip (done)", stage=st)
            continue
        t0 = time.time()
        m["stages"][st] = {"status": "running", "digest": dig, "started": t0}
        c.save_manifest(m)
        try:
            outs = STAGE_FNS[st](c, m)
        except Exception as e:
            m["stages"][st].update(status="failed", error=repr(e)[:2000])
            c.save_manifest(m)
            raise
        m["stages"][st].update(status="done", outputs=outs, seconds=round(time.time() - t0, 1))
        c.save_manifest(m)
        if st in ("soup", "eval"):
            retention_check(c, m, generate_factory)
            c.save_manifest(m)
        marker = c.out_dir / "PAUSE_AFTER"
        if marker.exists() and marker.read_text().strip() == st:
            marker.unlink()
            log.info("paused at stage boundary", stage=st)
            m["paused_after"] = st
            c.save_manifest(m)
            break
    return m


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore campaign")
    ap.add_argument("--out", required=True)
    ap.add_argument("--base-model", required=True)
    ap.add_argument("--stages", default="", help="comma list (default: all)")
    ap.add_argument("--force", default="")
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--gpu-ids", default="", help="comma list; 'auto' picks free GPUs")
    ap.add_argument("--config", action="append", default=[], help="stage=path.json overrides")
    ap.add_argument("--teacher", default="stub")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    ids = None
    if a.gpu_ids == "auto":
        from .nodes import pick_free_gpus
        ids = pick_free_gpus(a.gpus)
    elif a.gpu_ids:
        ids = [int(x) for x in a.gpu_ids.split(",")]
    cfgs = {}
    for kv in a.config:
        st, p = kv.split("=", 1)
        cfgs[st] = json.loads(Path(p).read_text())
    c = Campaign(Path(a.out), a.base_model, gpus=a.gpus, gpu_ids=ids, configs=cfgs, dry_run=a.dry_run,
                 teacher=a.teacher)
    m = run(c, [s for s in a.stages.split(",") if s] or None, [s for s in a.force.split(",") if s])
    print(json.dumps({k: v.get("status") for k, v in m["stages"].items()}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
