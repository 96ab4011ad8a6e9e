"""Reference arm of bench.py: the reference's SFT step on its own software stack.

The reference trains SFT through TRL ``SFTTrainer`` on ``accelerate`` FSDP
(kore/policy/sft.py:246-415, configs/accelerate_fsdp.yaml). Neither ``trl``
nor ``accelerate`` is installed in this offline image, so the reference's own
entry point cannot run. This module is the "reference-equivalent" arm: the
same model class, the same parallelism settings and the same per-step work,
built directly from the libraries those wrappers call, and nothing of
kore_b200 (no model, kernel or engine of this repository is imported):

* model: Hugging Face ``transformers`` ``Qwen3ForCausalLM`` built from a
  Qwen3-14B-architecture config, random init, SDPA attention
  (``preferred_attn_impl`` falls back to SDPA when no FlashAttention-2 wheel
  matches the GPU; on B200 SDPA dispatches to cuDNN / flash kernels);
* sharding: torch FSDP1 FULL_SHARD, one unit per ``Qwen3DecoderLayer``,
  ``backward_prefetch=BACKWARD_PRE``, ``forward_prefetch=True``,
  ``use_orig_params=True``, ``limit_all_gathers=True``, the settings that
  ``build_fsdp_kwargs`` returns (kore/policy/configs.py:580-651), read from the
  installed reference package when it is importable;
* precision: fp32 master parameters (what accelerate's FSDP prepare produces
  from a bf16 model under ``mixed_precision: bf16``), bf16 compute, bf16
  gradient reduce-scatter;
* activation checkpointing: HF layer-internal, ``use_reentrant=True``;
* optimizer: torch AdamW (fused), grad-norm clip 1.0 (HF Trainer defaults);
* loss: HF's mean token cross-entropy with labels = -100 on the first half of
  every sequence; micro-batch 2 (the reference's ``per_device_train_batch_size``)
  with gradient accumulation up to the bench's sequences per GPU.

Every step copies its token block from pinned host memory and reads the loss
back, as the HF Trainer's data loader and logging do.
"""
from __future__ import annotations

import json
import os
import sys
import time

REF_PKG = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")


def _fsdp_settings() -> dict:
    """The reference's FSDP kwargs (from baseline/_ref when importable)."""
    cfg = {"backward_prefetch": "backward_pre", "forward_prefetch": True, "use_orig_params": True,
           "limit_all_gathers": True, "transformer_layer_cls_to_wrap": ["Qwen3DecoderLayer"],
           "source": "built-in copy of kore/policy/configs.py:580-651 settings"}
    if os.path.isdir(os.path.join(REF_PKG, "kore")):
        sys.path.insert(0, REF_PKG)
        try:
            from types import SimpleNamespace

            from kore.policy.configs import build_fsdp_kwargs
            kw = build_fsdp_kwargs(SimpleNamespace(distributed=True, use_lora=False, model_id="Qwen/Qwen3-14B",
                                                   fsdp="full_shard auto_wrap", fsdp_cpu_offload=False,
                                                   fsdp_transformer_layer_cls=None))
            fc = kw["fsdp_config"]
            cfg = {k: fc[k] for k in ("backward_prefetch", "forward_prefetch", "use_orig_params",
                                       "limit_all_gathers", "transformer_layer_cls_to_wrap")}
            cfg["fsdp"] = kw["fsdp"]
            cfg["source"] = "baseline/_ref kore.policy.configs.build_fsdp_kwargs"
        except Exception as e:  # noqa: BLE001 - fall back to the recorded settings
            cfg["source_error"] = repr(e)
        finally:
            sys.path.remove(REF_PKG)
    return cfg


def run(args, clock_sampler_cls) -> None:
    import torch
    import torch.distributed as dist
    from torch.distributed.fsdp import BackwardPrefetch, MixedPrecision, ShardingStrategy
    from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
    from torch.distributed.fsdp.wrap import transformer_auto_wrap_policy
    import functools
    import transformers
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3DecoderLayer, Qwen3RotaryEmbedding

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    fs = _fsdp_settings()

    cfg = Qwen3Config(vocab_size=151936, hidden_size=5120, intermediate_size=17408, num_hidden_layers=40,
                      num_attention_heads=40, num_key_value_heads=8, head_dim=128,
                      max_position_embeddings=40960, rope_theta=1e6, rms_norm_eps=1e-6,
                      tie_word_embeddings=False, use_cache=False)
    if args.layers:
        cfg.num_hidden_layers = args.layers
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)   # fp32 parameters: the FSDP master
    model.config.use_cache = False

    def init_fn(module):
        meta = [t for t in list(module.parameters(recurse=False)) + list(module.buffers(recurse=False))
                if t.is_meta]
        if not meta:
            return
        module.to_empty(device=dev, recurse=False)
        with torch.no_grad():
            if isinstance(module, Qwen3RotaryEmbedding):
                fn = getattr(module, "rope_init_fn", None)
                if fn is None:
                    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
                    fn = (module.compute_default_rope_parameters if module.rope_type == "default"
                          else ROPE_INIT_FUNCTIONS[module.rope_type])
                inv, _ = fn(module.config, dev)
                module.inv_freq.copy_(inv)
                module.original_inv_freq.copy_(inv)
                return
            for name, p in module.named_parameters(recurse=False):
                if "norm" in type(module).__name__.lower():
                    p.fill_(1.0)
                else:
                    p.normal_(0.0, 0.02)

    wrap = functools.partial(transformer_auto_wrap_policy, transformer_layer_cls={Qwen3DecoderLayer})
    bp = {"backward_pre": BackwardPrefetch.BACKWARD_PRE, "backward_post": BackwardPrefetch.BACKWARD_POST}
    status = {"impl": "reference", "reference_class": "equivalent"}
    try:
        model = FSDP(model, sharding_strategy=ShardingStrategy.FULL_SHARD, auto_wrap_policy=wrap,
                     mixed_precision=MixedPrecision(param_dtype=torch.bfloat16, reduce_dtype=torch.bfloat16,
                                                    buffer_dtype=torch.bfloat16),
                     backward_prefetch=bp.get(str(fs["backward_prefetch"]).lower(), BackwardPrefetch.BACKWARD_PRE),
                     forward_prefetch=bool(fs["forward_prefetch"]), limit_all_gathers=bool(fs["limit_all_gathers"]),
                     use_orig_params=bool(fs["use_orig_params"]), device_id=dev, param_init_fn=init_fn,
                     sync_module_states=False)
        model.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": True})
        model.enable_input_require_grads()
        opt = torch.optim.AdamW(model.parameters(), lr=1e-5, betas=(0.9, 0.999), weight_decay=0.0, fused=True)
    except torch.OutOfMemoryError as e:
        _unavailable(rank, f"out of memory while sharding the fp32-master 14B model on {world} GPU(s): "
                           f"{str(e).splitlines()[0][:200]}")
        return

    B, S = args.seqs_per_gpu, args.seq
    mb = min(2, B)
    g = torch.Generator().manual_seed(1234 + rank)
    ids_host = torch.randint(0, cfg.vocab_size, (B, S), generator=g).pin_memory()
    lab_host = ids_host.clone()
    lab_host[:, : S // 2] = -100          # loss on the last 50% of each sequence
    lab_host = lab_host.pin_memory()

    def step():
        ids = ids_host.to(dev, non_blocking=True)
        lab = lab_host.to(dev, non_blocking=True)
        nacc = (B + mb - 1) // mb
        tot = torch.zeros((), device=dev)
        for s in range(0, B, mb):
            out = model(input_ids=ids[s:s + mb], labels=lab[s:s + mb], use_cache=False)
            (out.loss / nacc).backward()
            tot += out.loss.detach() / nacc
        model.clip_grad_norm_(1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return tot

    try:
        model.train()
        for _ in range(args.warmup):
            float(step().item())
        torch.cuda.synchronize()
        dist.barrier()
        clk = clock_sampler_cls(local).start()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(args.steps):
            loss = float(step().item())
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1000 / args.steps
        clocks = clk.stop()
    except torch.OutOfMemoryError as e:
        _unavailable(rank, f"out of memory in the training step on {world} GPU(s): "
                           f"{str(e).splitlines()[0][:200]}")
        return
    ms_t = torch.tensor([e0.elapsed_time(e1) / args.steps, wall], device=dev)
    dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, wall_ms = float(ms_t[0]), float(ms_t[1])
    tokens = B * S * world
    if rank == 0:
        status.update({
            "metric": "sft_tokens_per_s", "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform-random token ids, random-init weights",
            "config": {"model": "qwen3-14b-arch (dense)", "layers": cfg.num_hidden_layers,
                       "global_batch": B * world, "seq_len": S, "parallelism": f"fsdp{world}-full_shard",
                       "micro_batch": mb, "loss": "last 50% of each sequence",
                       "optimizer": "torch AdamW (fused), fp32 master", "checkpointing": "HF reentrant",
                       "attention": "sdpa", "fsdp_settings": fs,
                       "stack": f"torch {torch.__version__}, transformers {transformers.__version__} "
                                "(reference pins 4.57.6 + trl 0.29.1 + accelerate 1.14.0; trl/accelerate "
                                "not installable offline)",
                       "l2": "inputs larger than L2 (weights and optimizer state streamed per step)"},
            "loss": loss, "clocks": clocks, "gpu_launches": None,
            "e2e": {"value": tokens / (wall_ms / 1000.0), "unit": "tokens/s", "ms_per_step": wall_ms,
                    "h2d_bytes_per_step": int(ids_host.numel() * 8 * 2), "d2h_bytes_per_step": 4},
            "memory": {"peak_allocated_gb": round(torch.cuda.max_memory_allocated() / 1e9, 2)},
        })
        print(json.dumps(status), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def _unavailable(rank: int, why: str) -> None:
    if rank == 0:
        print(json.dumps({"impl": "reference", "reference_class": "equivalent", "unavailable": why}), flush=True)
