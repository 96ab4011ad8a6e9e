"""Headline benchmark: SFT tokens/s of the Qwen3-14B-architecture dense model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kore|reference]

For N > 1 run under ``python -m torch.distributed.run --nproc-per-node N``.
Config (SFT row): 40 layers, hidden 5120, 40 Q / 8 KV heads,
head_dim 128, FFN 17408, vocab 151936, RoPE 1e6; random-init bf16 weights,
fp32 AdamW moments; packed sequences of 8192 uniform-random token ids, loss
on the last 50% of each sequence; 8 sequences per GPU per step (global batch
64 on 8 GPUs, weak scaling).

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
torch.cuda.synchronize and CUDA events on the launching stream; the step
time is the max over ranks. Every step streams all 29.5 GB of weights plus
optimizer state, far larger than the 126 MB L2, so no explicit flush is
needed. A second timed loop (``e2e``) calls the public API
``CausalLMTrainer.train_step`` with pinned host inputs and reads the loss
back each step.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

if any(a in ("grpo", "dpo", "--metric=grpo", "--metric=dpo") for a in sys.argv) and "reference" not in sys.argv:
    # the GRPO / DPO phases free and re-allocate tens of GB in blocks of
    # different sizes every step (KV cache, gradients, reference layers):
    # growable segments keep that from fragmenting the 180 GB
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sft_tokens_per_s"
BASELINE_VALUE = None  # the reference publishes no SFT tokens/s figure


class ClockSampler:
    """Samples SM clocks and throttle reasons of the visible GPUs via NVML
    while the timed region runs (read-only queries)."""

    def __init__(self, index: int, period_s: float = 0.2):
        self.index = index
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return self
        names = {
            "hw_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(pynvml, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(pynvml, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for n, bit in names.items():
                        if r & bit:
                            self.reasons.add(n)
                except Exception:
                    pass
                self._stop.wait(self.period)

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def stop(self) -> dict:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)
        s = sorted(self.samples)
        med = s[len(s) // 2] if s else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(s)}


def reference_arm(args) -> None:
    """The reference's SFT step on its own stack.

    The reference's entry point (TRL SFTTrainer over accelerate FSDP) needs
    ``trl`` and ``accelerate``; when they are missing, the reference-equivalent
    arm in ``baseline/reference_arm.py`` runs the same model class, FSDP
    settings, precision, checkpointing and loss on plain torch + transformers
    (none of kore_b200 is imported on that path)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    why = None
    if not os.path.isdir(os.path.join(ref, "kore")):
        why = "reference not installed at baseline/_ref"
    else:
        probe = subprocess.run(
            [sys.executable, "-c",
             "import sys; sys.path.insert(0, %r); import kore.policy.sft as s; "
             "import trl, accelerate" % ref],
            capture_output=True, text=True)
        if probe.returncode != 0:
            last = (probe.stderr.strip().splitlines() or ["import failed"])[-1]
            why = "TRL SFTTrainer over accelerate FSDP cannot run offline: " + last
    if why is None:
        raise SystemExit("reference arm: trl + accelerate importable; run the reference's "
                         "kore.policy.sft entry point directly")
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import reference_arm as ra
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "note": "unmodified entry point unavailable (" + why
                          + "); running the reference-equivalent arm"}), file=sys.stderr, flush=True)
    ra.run(args, ClockSampler)


def _recompute_note(trainer, cfg) -> str:
    L = cfg.num_hidden_layers
    sh = getattr(trainer, "_shuttle", None)
    if sh is not None and sh.keep_mid is not None:
        return (f"second moments in pinned host memory during micro-batches 2..{sh.n - 1} (copied out and back on "
                f"a side stream, overlapped with the first and last micro-batch); those micro-batches keep "
                f"{sh.keep_mid} of {L} layer contexts, the first and last recompute all {L}")
    return f"{L - trainer.eng.keep_layers} of {L} layers recompute their GEMMs"


def grpo_main(args) -> None:
    """GRPO-step tokens/s (BASELINE GRPO row): multi-turn rollout + reference
    log-probs + update + weight sync, one optimizer step per GRPO step.

    Weak scaling: every GPU rolls 8 prompts x group 8 = 64 trajectories (at
    N = 8 that is the 64 x 8 of the BASELINE config), 1024-token prompts, 3
    turns of up to 2048 sampled tokens (temperature 1.0) with 32 feedback
    tokens between turns, synthetic per-turn rewards {0, 0.1, 0.3} + 0.9 Phi' -
    Phi, clip 0.2, KL beta 0.01 against a frozen reference copy. Tokens counted
    = every trajectory's final transcript (prompt + generations + feedback)."""
    import torch

    from kore_b200 import ops
    from kore_b200.env.base import SyntheticRewardEnv
    from kore_b200.models import PRESETS, Qwen3Weights
    from kore_b200.parallel.dist import init_distributed
    from kore_b200.policy.configs import GRPOConfig
    from kore_b200.policy.grpo import GRPOTrainer

    assert args.warmup >= 3, "at least 3 warm-up steps"
    ctx = init_distributed()
    cfg = PRESETS[args.model]()
    if args.layers:
        cfg.num_hidden_layers = args.layers
    ops.native()
    W = ctx.world
    G = 8
    gc = GRPOConfig(num_trajectories=G, num_turns=args.turns, tasks_per_step=8 * W,
                    max_response_length=args.gen_len, max_prompt_length=16384, max_feedback_tokens=32,
                    learning_rate=1e-6, temperature=1.0, top_p=1.0, clip_ratio_low=0.2, clip_ratio_high=0.2,
                    ref_anchor_coef=0.01, dynamic_sampling=False, starpo_s=False, bf16=True,
                    overlong_mask=False, total_steps=args.warmup + args.steps, kv_page_size=64,
                    reward_env="synthetic", seed=0, offload_state=args.offload)
    gc.comm = args.comm
    gc.rollout_parallel = args.rollout_parallel
    env = SyntheticRewardEnv(seed=0, prompt_len=args.prompt_len, feedback_len=32, vocab_size=cfg.vocab_size)
    w = Qwen3Weights(cfg, device=ctx.device, dtype=torch.bfloat16, seed=0, pad_multiple=128 * max(1, W))
    tr = GRPOTrainer(gc, weights=w, env=env, ctx=ctx,
                     rollout_kwargs=dict(max_batch=G * 8, page_size=64, max_seq_len=16384))
    del w
    tasks = [f"synthetic-{i}" for i in range(8 * W)]
    for _ in range(args.warmup):
        st = tr.train_step(tasks, micro_batch_tokens=args.micro_tokens)
    torch.cuda.synchronize()
    ctx.barrier()
    ops.reset_launch_count()
    clk = ClockSampler(ctx.local_rank).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    toks, phases = 0, {}
    for _ in range(args.steps):
        st = tr.train_step(tasks, micro_batch_tokens=args.micro_tokens)
        toks += st["traj_tokens"]
        for k, v in st.items():
            if k.startswith("ms_"):
                phases[k[3:]] = phases.get(k[3:], 0.0) + v / args.steps
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1000 / args.steps
    clocks = clk.stop()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1) / args.steps)
    wall_ms = ctx.max_over_ranks(wall)
    t = torch.tensor([float(toks) / args.steps], device=ctx.device)
    ctx.all_reduce(t)
    tokens = float(t.item())
    if ctx.is_main:
        print(json.dumps({
            "metric": "grpo_step_tokens_per_s", "value": tokens / (ms / 1000.0), "unit": "tokens/s",
            "n_gpus": W, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform-random prompts and feedback, synthetic rewards, random-init weights",
            "config": {"model": "qwen3-14b-arch (dense)" if args.model == "qwen3-14b" else args.model,
                       "layers": cfg.num_hidden_layers, "prompts": 8 * W, "group": G,
                       "trajectories_per_gpu": 8 * G, "prompt_len": args.prompt_len, "turns": args.turns,
                       "max_new_per_turn": args.gen_len, "feedback_tokens": 32,
                       "tokens_per_step": tokens, "gen_tokens_per_step_rank0": st["gen_tokens"],
                       "parallelism": (f"dp{W} replicated rollout" if W == 1 or args.rollout_parallel == "replica"
                                       else f"tp{W} rollout") + (f", zero2-{args.comm}" if W > 1 else ""),
                       "clip": 0.2, "kl_beta": 0.01, "temperature": 1.0,
                       "offload": {"optimizer_state_gb_parked": st.get("offload_opt_gb"),
                                   "gradients_dropped_during_rollout": st.get("dropped_grads"),
                                   "reference_model": tr.ref_placement},
                       "l2": "inputs larger than L2 (weights and KV cache streamed every decode step)"},
            "phases_ms": phases, "clocks": clocks, "gpu_launches": ops.launch_count(),
            "e2e": {"value": tokens / (wall_ms / 1000.0), "unit": "tokens/s", "ms_per_step": wall_ms,
                    "h2d_bytes_per_step": int(8 * W * G * (args.prompt_len + 32 * (args.turns - 1)) * 8 / W),
                    "d2h_bytes_per_step": int(8 * G * (args.turns * args.gen_len) * 12)},
            "memory": {"peak_allocated_gb": round(torch.cuda.max_memory_allocated() / 1e9, 2)},
            "impl": "kore"}), flush=True)


def dpo_main(args) -> None:
    """DPO tokens/s (BASELINE DPO row), weak-scaled: 4 chosen/rejected pairs per
    GPU (32 on 8 GPUs), a shared 1024-token prompt + 3072-token responses of
    uniform-random ids, beta 0.1, sigmoid loss; the frozen reference is
    sharded over the ranks (streamed from host memory on one GPU)."""
    import torch

    from kore_b200 import ops
    from kore_b200.models import PRESETS, Qwen3Weights
    from kore_b200.parallel.dist import init_distributed
    from kore_b200.policy.configs import DPOConfig
    from kore_b200.policy.dpo import DPOTrainer

    assert args.warmup >= 3, "at least 3 warm-up steps"
    ctx = init_distributed()
    cfg = PRESETS[args.model]()
    if args.layers:
        cfg.num_hidden_layers = args.layers
    ops.native()
    W = ctx.world
    P, R = args.prompt_len, args.response_len
    dc = DPOConfig(beta=0.1, learning_rate=1e-6, lr_scheduler_type="constant", warmup_ratio=0.0, bf16=True,
                   use_lora=False, micro_pairs=1, ref_placement=args.ref_placement)
    dc.comm = args.comm
    w = Qwen3Weights(cfg, device=ctx.device, dtype=torch.bfloat16, seed=0, pad_multiple=128 * max(1, W))
    dt = DPOTrainer(dc, ctx, w, total_steps=args.warmup + args.steps)   # reference = the policy at step 0
    del w
    g = torch.Generator().manual_seed(77 + ctx.rank)

    def batch():
        out = []
        for _ in range(args.pairs_per_gpu):
            prompt = torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist()
            pair = []
            for _ in range(2):
                pair.append((prompt + torch.randint(0, cfg.vocab_size, (R,), generator=g).tolist(), P))
            out.append(pair)
        return out

    batches = [batch() for _ in range(min(4, args.warmup + args.steps))]
    for i in range(args.warmup):
        dt.step(batches[i % len(batches)])
    torch.cuda.synchronize()
    ctx.barrier()
    ops.reset_launch_count()
    clk = ClockSampler(ctx.local_rank).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for i in range(args.steps):
        loss = dt.step(batches[(args.warmup + i) % len(batches)])
    e1.record()
    torch.cuda.synchronize()
    wall_ms = ctx.max_over_ranks((time.perf_counter() - t0) * 1000 / args.steps)
    clocks = clk.stop()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1) / args.steps)
    tokens = args.pairs_per_gpu * 2 * (P + R) * W
    if ctx.is_main:
        print(json.dumps({
            "metric": "dpo_tokens_per_s", "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": W,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform-random prompt/response ids, random-init weights",
            "config": {"model": "qwen3-14b-arch (dense)" if args.model == "qwen3-14b" else args.model,
                       "layers": cfg.num_hidden_layers, "pairs": args.pairs_per_gpu * W, "prompt_len": P,
                       "response_len": R, "beta": 0.1, "loss": "sigmoid",
                       "reference_model": dt.ref_placement,
                       "parallelism": f"dp{W}" + (f"-zero2-{args.comm}" if W > 1 else ""),
                       "l2": "inputs larger than L2 (weights streamed every micro-batch)"},
            "loss": loss, "clocks": clocks, "gpu_launches": ops.launch_count(),
            "e2e": {"value": tokens / (wall_ms / 1000.0), "unit": "tokens/s", "ms_per_step": wall_ms,
                    "h2d_bytes_per_step": int(args.pairs_per_gpu * 2 * (P + R) * 8),
                    "d2h_bytes_per_step": 8},
            "memory": {"peak_allocated_gb": round(torch.cuda.max_memory_allocated() / 1e9, 2)},
            "impl": "kore"}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kore", choices=["kore", "reference"])
    ap.add_argument("--model", default="qwen3-14b")
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--seqs-per-gpu", type=int, default=8)
    ap.add_argument("--micro-batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="debug only: override layer count")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--metric", default="sft", choices=["sft", "grpo", "dpo"])
    ap.add_argument("--pairs-per-gpu", type=int, default=4, help="dpo: chosen/rejected pairs per GPU")
    ap.add_argument("--response-len", type=int, default=3072, help="dpo: response tokens")
    ap.add_argument("--ref-placement", default="auto", choices=["auto", "resident", "host", "shard"],
                    help="dpo: where the frozen reference's layers live")
    ap.add_argument("--turns", type=int, default=3, help="grpo: turns per trajectory")
    ap.add_argument("--gen-len", type=int, default=2048, help="grpo: max sampled tokens per turn")
    ap.add_argument("--prompt-len", type=int, default=1024, help="grpo: prompt tokens")
    ap.add_argument("--rollout-parallel", default="replica", choices=["replica", "tp"],
                    help="grpo, several GPUs: each rank decodes its own rows, or heads split over ranks")
    ap.add_argument("--micro-tokens", type=int, default=8192, help="grpo: tokens per update micro-batch")
    ap.add_argument("--offload", default="auto", choices=["auto", "always", "never"],
                    help="grpo: park optimizer state / reference model in host memory between phases")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl", "nvls"],
                    help="data plane of the sharded optimizer (N > 1)")
    ap.add_argument("--recompute", default="auto", choices=["auto", "full", "none"],
                    help="activation recompute: auto keeps whole layers' contexts while HBM allows")
    ap.add_argument("--zero", type=int, default=2, choices=[2, 3],
                    help="2: resident params, sharded grads/optimizer; 3: decoder layers fully sharded")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        if args.metric != "sft":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference's GRPO loop needs trl + "
                                  "accelerate (not installable offline); only the SFT arm has an equivalent"}))
            return None
        return reference_arm(args)
    if args.metric == "grpo":
        return grpo_main(args)
    if args.metric == "dpo":
        return dpo_main(args)

    import torch

    from kore_b200 import ops
    from kore_b200.engine.trainer import CausalLMTrainer
    from kore_b200.models import PRESETS
    from kore_b200.parallel.dist import init_distributed

    assert args.warmup >= 3, "at least 3 warm-up steps"
    ctx = init_distributed()
    assert ctx.world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {ctx.world}"
    cfg = PRESETS[args.model]()
    if args.layers:
        cfg.num_hidden_layers = args.layers
    ops.native()  # fail loudly if the extension is missing
    trainer = CausalLMTrainer(cfg, ctx, lr=1e-5, max_grad_norm=1.0, seed=0,
                              micro_batch_size=args.micro_batch,
                              comm=args.comm, zero_stage=args.zero,
                              recompute=args.recompute)
    B, S = args.seqs_per_gpu, args.seq
    g = torch.Generator().manual_seed(1234 + ctx.rank)
    # a fresh token block every step (cycled over NB distinct blocks)
    NB = max(2, min(8, args.steps + args.warmup))
    ids_hosts = [torch.randint(0, cfg.vocab_size, (B, S), generator=g).pin_memory() for _ in range(NB)]
    mask_host = torch.zeros(B, S, dtype=torch.bool)
    mask_host[:, S // 2:] = True  # loss on the last 50% of each sequence
    mask_host = mask_host.pin_memory()
    ids_devs = [h.cuda() for h in ids_hosts]
    ids_host = ids_hosts[0]
    mask = mask_host.cuda()

    for i in range(args.warmup):
        trainer.train_step_device(ids_devs[i % NB], mask)
    torch.cuda.synchronize()
    ctx.barrier()

    # ---------------- device-timed loop
    ops.reset_launch_count()
    clk = ClockSampler(ctx.local_rank).start()
    ctx.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        loss = trainer.train_step_device(ids_devs[(args.warmup + i) % NB], mask)
    e1.record()
    torch.cuda.synchronize()
    ctx.barrier()
    clocks = clk.stop()
    launches = ops.launch_count()
    mstats = torch.cuda.memory_stats()
    memory = {"peak_allocated_gb": round(torch.cuda.max_memory_allocated() / 1e9, 2),
              "reserved_gb": round(torch.cuda.memory_reserved() / 1e9, 2),
              "alloc_retries": int(mstats.get("num_alloc_retries", 0)),
              "device_mallocs": int(mstats.get("num_device_alloc", 0)),
              "device_frees": int(mstats.get("num_device_free", 0))}
    dev_ms = e0.elapsed_time(e1) / args.steps
    ms = ctx.max_over_ranks(dev_ms)
    loss_v = float(loss.item())

    # ---------------- end-to-end loop through the public API
    e2e = None
    if not args.no_e2e:
        torch.cuda.synchronize()
        ctx.barrier()
        t0 = time.perf_counter()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for i in range(args.steps):
            trainer.train_step(ids_hosts[i % NB], mask_host)
        s1.record()
        torch.cuda.synchronize()
        e2e_ms = ctx.max_over_ranks(s0.elapsed_time(s1) / args.steps)
        wall_ms = ctx.max_over_ranks((time.perf_counter() - t0) * 1000 / args.steps)
        tok = B * S * ctx.world
        e2e = {"value": tok / (e2e_ms / 1000.0), "unit": "tokens/s",
               "ms_per_step": e2e_ms, "wall_ms_per_step": wall_ms,
               "h2d_bytes_per_step": int(ids_host.numel() * ids_host.element_size()
                                         + mask_host.numel() * mask_host.element_size()),
               "d2h_bytes_per_step": 4}

    tokens = B * S * ctx.world
    value = tokens / (ms / 1000.0)
    if ctx.is_main:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ctx.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None,
            "dtype": "bf16", "data": f"synthetic uniform-random token ids ({NB} distinct blocks cycled), random-init weights",
            "config": {"model": "qwen3-14b-arch (dense)" if args.model == "qwen3-14b" else args.model,
                       "layers": cfg.num_hidden_layers,
                       "global_batch": B * ctx.world, "seq_len": S,
                       "parallelism": f"dp{ctx.world}" + (
                           (f"-zero2-{args.comm}" if args.zero == 2 else
                            ("-zero3-copy-engine-gathers" if args.comm == "fused" else "-zero3-nccl"))
                           if ctx.world > 1 else ""),
                       "loss": "last 50% of each sequence", "micro_batch": args.micro_batch,
                       "optimizer": f"AdamW fp32 moments, master={trainer.master_mode}",
                       "activation_recompute": _recompute_note(trainer, cfg),
                       "l2": "inputs larger than L2 (29.5 GB of weights streamed per step)"},
            "loss": loss_v, "clocks": clocks, "gpu_launches": launches, "e2e": e2e, "memory": memory,
            "impl": "kore",
        }
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
