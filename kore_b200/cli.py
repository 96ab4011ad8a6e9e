"""``kore`` command line (subcommands mirror the reference's CLI,
kore/cli.py:187-259, plus midtrain / soup / bench / launch).

    kore tasks [--split train|heldout]
    kore sft|dpo|grpo|midtrain <config.json>
    kore soup --base DIR --kore DIR --out DIR [--alpha A]
    kore datagen {repair,groups,wins,evolve} ...
    kore build-datasets {sft,dpo,rft} ...
    kore value-train ...
    kore study --tasks A,B --out p0.json | kore residual-transfer p0.json | kore calibrate
    kore eval ...
    kore bench [--gpus N ...]
    kore launch <stage> <config.json> [--gpus N] [--dry-run]
    kore campaign --out DIR --base-model M [--stages ...]
    kore supervise -- <cmd ...>
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path
from typing import List, Optional

STAGES = {"sft": "kore_b200.policy.sft", "dpo": "kore_b200.policy.dpo", "grpo": "kore_b200.policy.grpo",
          "midtrain": "kore_b200.policy.midtrain"}


def launch_command(stage: str, cfg_path: str, gpus: int, port: int = 29511) -> List[str]:
    """torchrun command of a stage (the reference's accelerate launcher,
    scripts/launch_distributed.sh:76-112)."""
    if stage not in STAGES:
        raise SystemExit(f"unknown stage {stage!r}; expected one of {sorted(STAGES)}")
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr=127.0.0.1", f"--master-port={port}", "-m", STAGES[stage], cfg_path]


def cmd_stage(args) -> int:
    import importlib
    return importlib.import_module(STAGES[args.cmd])._main([args.config])


def cmd_launch(args) -> int:
    cmd = launch_command(args.stage, args.config, args.gpus, args.port)
    if args.dry_run:
        print(" ".join(cmd))
        return 0
    return subprocess.call(cmd)


def cmd_tasks(args) -> int:
    from .tasks.registry import all_tasks, split_tasks
    if getattr(args, "audit", False):
        from .tasks.audit import main as audit_main
        return audit_main([])
    if args.split:
        tr, ho = split_tasks(seed=args.seed)
        ids = tr if args.split == "train" else ho
    else:
        ids = [t.task_id for t in all_tasks()]
    for t in ids:
        print(t if isinstance(t, str) else t.task_id)
    return 0


def cmd_soup(args) -> int:
    from .policy.configs import SoupConfig
    from .policy.soup import build_soup
    cfg = SoupConfig(base_model_id=args.base, kore_checkpoint=args.kore, output_dir=args.out,
                     alphas=tuple(args.alpha or (0.7, 0.8, 0.9)))
    print(json.dumps(build_soup(cfg)))
    return 0


def cmd_bench(args, rest) -> int:
    root = Path(__file__).resolve().parent.parent
    return subprocess.call([sys.executable, str(root / "bench.py")] + rest)


def cmd_datagen(args, rest) -> int:
    from .data import factory
    return factory.main([args.kind] + rest)


def cmd_build(args, rest) -> int:
    from .data import build_datasets
    return build_datasets.main([args.kind] + rest)


def cmd_value(args, rest) -> int:
    from .value import replay_train
    return replay_train.main(rest)


def cmd_eval(args, rest) -> int:
    """``kore eval --model ...`` (fast_p on a split) or ``kore eval vs-frontier ...``
    (head-to-head against a frontier model)."""
    if rest and rest[0] == "vs-frontier":
        from .eval import vs_frontier
        return vs_frontier.main(rest[1:])
    from .eval import cli as ecli
    return ecli.main(rest)


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="kore", description="KORE on B200: post-training for GPU-kernel RL")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for st in STAGES:
        p = sub.add_parser(st, help=f"run the {st} stage from a JSON config")
        p.add_argument("config")
    p = sub.add_parser("launch", help="torchrun a stage on N GPUs")
    p.add_argument("stage")
    p.add_argument("config")
    p.add_argument("--gpus", type=int, default=8)
    p.add_argument("--port", type=int, default=29511)
    p.add_argument("--dry-run", action="store_true")
    p = sub.add_parser("tasks", help="list kernel tasks")
    p.add_argument("--split", choices=["train", "heldout"])
    p.add_argument("--audit", action="store_true", help="data-scale report of the corpus")
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("soup", help="WiSE-FT interpolation")
    p.add_argument("--base", required=True)
    p.add_argument("--kore", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--alpha", type=float, nargs="*")
    sub.add_parser("bench", help="headline benchmark (bench.py)")
    p = sub.add_parser("datagen", help="data factory generators")
    p.add_argument("kind", choices=["repair", "groups", "wins", "evolve", "agentic", "qa"])
    p = sub.add_parser("build-datasets", help="assemble SFT / DPO / RFT datasets")
    p.add_argument("kind", choices=["sft", "dpo", "rft"])
    sub.add_parser("value-train", help="train the kernel value model")
    sub.add_parser("eval", help="evaluation suite")
    sub.add_parser("campaign", help="staged campaign with a resumable manifest")
    sub.add_parser("supervise", help="relaunch-with-resume supervisor / monitor")
    sub.add_parser("proof", help="smokes and proofs (env, sft, grpo, breadth, ops, grpo-repro)")
    sub.add_parser("study", help="speed-of-light study (eta vs speedup, residual model, monotone valley)")
    sub.add_parser("residual-transfer", help="does the residual model transfer across families")
    sub.add_parser("study-plots", help="SVG figures of a study report")
    sub.add_parser("calibrate", help="measure HBM copy and bf16 GEMM peaks on this GPU")
    return ap


def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    ap = build_parser()
    args, rest = ap.parse_known_args(argv)
    if args.cmd in STAGES:
        return cmd_stage(args)
    return {"launch": lambda: cmd_launch(args), "tasks": lambda: cmd_tasks(args),
            "soup": lambda: cmd_soup(args), "bench": lambda: cmd_bench(args, rest),
            "datagen": lambda: cmd_datagen(args, rest), "build-datasets": lambda: cmd_build(args, rest),
            "value-train": lambda: cmd_value(args, rest), "eval": lambda: cmd_eval(args, rest),
            "proof": lambda: __import__("kore_b200.proofs", fromlist=["main"]).main(rest),
            "study": lambda: __import__("kore_b200.analysis.p0_runner", fromlist=["main"]).main(rest),
            "residual-transfer": lambda: __import__("kore_b200.analysis.residual_transfer",
                                                    fromlist=["main"]).main(rest),
            "study-plots": lambda: __import__("kore_b200.analysis.plots", fromlist=["main"]).main(rest),
            "calibrate": lambda: __import__("kore_b200.analysis.calibrate", fromlist=["main"]).main(rest),
            "campaign": lambda: __import__("kore_b200.campaign.orchestrator", fromlist=["main"]).main(rest),
            "supervise": lambda: __import__("kore_b200.campaign.supervise", fromlist=["main"]).main(rest)}[args.cmd]()


if __name__ == "__main__":
    raise SystemExit(main())
