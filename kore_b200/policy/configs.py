"""Stage configuration dataclasses (the public JSON schema of every trainer).

Field names and defaults are the reference's config schema
(kore/policy/configs.py:35-545) so the same ``configs/*.json`` files drive
these trainers; keys that only steered the reference's HF/accelerate/
DeepSpeed stack (``fsdp``, ``sharding_backend``, ``zero_stage``,
``synced_gpus``, ``fsdp_version``, ``ds_config``...) are accepted and mapped
onto this framework's own sharding plan. B200-specific knobs are added at the
end of each dataclass (tensor/expert parallel sizes, rollout engine sizes,
data plane of the fused collectives).

Everything here is torch-free so configs can be built and validated on CPU.
"""
from __future__ import annotations

import glob
import json
import os
from dataclasses import asdict, dataclass, field, fields
from typing import Optional

MODEL_14B = "Qwen/Qwen3-14B"
MODEL_32B = "Qwen/Qwen3-32B"


@dataclass
class LoRAConfig:
    r: int = 32
    lora_alpha: int = 64
    lora_dropout: float = 0.05
    bias: str = "none"
    task_type: str = "CAUSAL_LM"
    target_modules: list = field(default_factory=lambda: [
        "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"])


@dataclass
class DistributedMixin:
    """Multi-GPU knobs shared by every trainer.

    ``fsdp`` keeps the reference's sharding string: ``full_shard`` selects
    ZeRO-3-style per-unit parameter sharding (all-gather fused into the first
    consuming GEMM), ``shard_grad_op`` (or GRPO's default) keeps parameters
    resident and shards gradients + optimizer state (ZeRO-2).
    """
    distributed: bool = False
    fsdp: str = "full_shard auto_wrap"
    fsdp_transformer_layer_cls: Optional[str] = None
    fsdp_cpu_offload: bool = False
    dataloader_num_workers: int = 12
    dataloader_pin_memory: bool = True
    dataloader_prefetch_factor: int = 4
    dataset_num_proc: int = 32
    # --- B200 runtime knobs (not in the reference)
    comm: str = "nccl"                 # "nccl" | "fused": data plane of the sharded optimizer
    micro_batch_tokens: int = 0        # pack micro-batches up to this many tokens (0 = per sample)
    save_attention: bool = True        # selective activation checkpointing


@dataclass
class SFTConfig(DistributedMixin):
    model_id: str = MODEL_14B
    dataset_path: str = ""
    output_dir: str = "runs/sft"
    learning_rate: float = 1e-5
    lr_scheduler_type: str = "cosine"
    num_train_epochs: float = 3.0
    warmup_ratio: float = 0.03
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0
    per_device_train_batch_size: int = 4
    gradient_accumulation_steps: int = 4
    max_seq_length: int = 16384
    bf16: bool = True
    gradient_checkpointing: bool = True
    packing: bool = False
    assistant_only_loss: bool = True
    repair_loss_weight: float = 2.0
    use_lora: bool = True
    lora: LoRAConfig = field(default_factory=LoRAConfig)
    seed: int = 0
    logging_steps: int = 10
    save_steps: int = 200
    report_to: str = "none"
    max_steps: int = -1
    save_total_limit: int = 1


@dataclass
class DPOConfig(DistributedMixin):
    model_id: str = MODEL_14B
    ref_model_id: Optional[str] = None
    dataset_path: str = ""
    output_dir: str = "runs/dpo"
    beta: float = 0.1
    learning_rate: float = 5e-6
    lr_scheduler_type: str = "cosine"
    num_train_epochs: float = 1.0
    warmup_ratio: float = 0.03
    weight_decay: float = 0.0
    per_device_train_batch_size: int = 2
    gradient_accumulation_steps: int = 8
    max_length: int = 16384
    bf16: bool = True
    gradient_checkpointing: bool = True
    use_lora: bool = True
    lora: LoRAConfig = field(default_factory=LoRAConfig)
    seed: int = 0
    logging_steps: int = 10
    save_steps: int = 200
    report_to: str = "none"
    max_steps: int = -1
    max_prompt_length: int = 4096
    # --- B200 knobs (not in the reference)
    ref_placement: str = "auto"         # frozen reference: resident | host (streamed) | shard (all-gathered) | auto
    micro_pairs: int = 1                # pairs per forward/backward micro-batch


@dataclass
class GRPOConfig(DistributedMixin):
    model_id: str = MODEL_32B
    output_dir: str = "runs/grpo"
    num_trajectories: int = 16
    num_turns: int = 4
    serial_refine: bool = True
    tasks_per_step: int = 8
    correctness_weight: float = 0.3
    gamma: float = 0.4
    per_turn_as_sample: bool = True
    clip_ratio_low: float = 0.03
    clip_ratio_high: float = 0.04
    adv_eps: float = 1e-6
    ppo_epochs: int = 1
    overlong_mask: bool = True
    overlong_buffer_len: int = 512
    adaptive_steps: bool = False
    min_steps: int = 100
    plateau_patience: int = 40
    plateau_min_delta: float = 1e-3
    learning_rate: float = 2e-6
    lr_scheduler_type: str = "constant"
    warmup_ratio: float = 0.0
    max_grad_norm: float = 0.5
    total_steps: int = 500
    max_prompt_length: int = 16384
    max_response_length: int = 16384
    bf16: bool = True
    gradient_checkpointing: bool = True
    temperature: float = 0.9
    top_p: float = 1.0
    use_lora: bool = False
    sharding_backend: str = "auto"
    fsdp_version: int = 1
    zero_stage: int = 3
    cpu_offload: bool = False
    ds_config: Optional[str] = None
    synced_gpus: bool = True
    rc_grpo: bool = False
    rc_p_high: float = 0.5
    variance_floor: float = 0.1
    avspo_virtual_k: int = 2
    sc_grpo: bool = False
    sc_grpo_w_min: float = 0.5
    sc_grpo_w_max: float = 2.0
    gtpo_codesim: bool = False
    gtpo_codesim_scale: float = 0.3
    kevin_best_kernel_scoring: bool = True
    cot_masking: bool = True
    ref_checkpoint: Optional[str] = None
    ref_anchor_coef: float = 1e-3
    starpo_s: bool = True
    starpo_min_std: float = 1e-3
    starpo_keep_frac: float = 0.75
    dynamic_sampling: bool = True
    target_groups: Optional[int] = None
    max_sampling_attempts: Optional[int] = None
    coevolve: bool = False
    coevolve_batch: Optional[int] = None
    coevolve_include_vendor: bool = True
    coevolve_distill_path: Optional[str] = None
    coevolve_distill_min_speedup: float = 1.0
    value_prefilter: bool = False
    num_candidates_per_turn: int = 8
    value_prefilter_k: int = 4
    value_model_path: Optional[str] = None
    reward_phase: str = "all"
    reward_mode: str = "speedup"
    physics_weight: float = 1.0
    credit_incorrect_turns: bool = False
    physics_shaping_weight: float = 0.0
    use_search: bool = False
    search_budget: int = 64
    search_every: int = 25
    search_bnb: bool = False
    search_value_prior: bool = False
    search_k_expand: int = 4
    search_max_depth: Optional[int] = None
    roofline_gate: bool = False
    roofline_tol: float = 0.25
    physics_live_counters: bool = False
    transform_discover: bool = False
    coevolve_mint: bool = False
    coevolve_mint_batch: int = 8
    coevolve_evolve_grammar: bool = False
    coevolve_regret_vs_opus: bool = False
    coevolve_opus_scores_path: Optional[str] = None
    adversarial_coevolve: bool = False
    agentic: bool = False
    tool_reward_weight: float = 0.2
    max_tool_turns: int = 8
    agentic_transform_tools: bool = False
    seed: int = 0
    logging_steps: int = 1
    save_steps: int = 50
    report_to: str = "none"
    # --- B200 rollout engine knobs (not in the reference)
    rollout_tp: int = 0                 # tensor-parallel size of the rollout engine (0 = world)
    rollout_max_batch: int = 512        # concurrent sequences in continuous batching
    kv_page_size: int = 128             # tokens per paged-KV page
    kv_cache_fraction: float = 0.35     # fraction of free HBM reserved for the KV pool
    reward_env: str = "kernel"          # "kernel" (KoreEnv) | "synthetic" (benchmark reward)
    batched_rollout: bool = True        # all groups of a step in one multi-turn batch (CUDA-graph decode)
    max_feedback_tokens: int = 1024     # per-turn feedback budget of the batched rollout
    pack_trajectories: bool = True      # train all turns of a trajectory in one packed sequence
    old_logp_source: str = "trainer"    # "trainer" (policy forward of the update) | "sampler"
    offload_state: str = "auto"         # optimizer state / frozen ref to host between phases: auto|always|never
    ref_placement: str = "auto"         # frozen KL reference: resident | host (streamed) | shard (all-gathered) | auto
    rollout_parallel: str = "replica"   # several GPUs: replica (each rank decodes its own rows) | tp (heads split)


@dataclass
class MidTrainConfig(DistributedMixin):
    model_id: str = MODEL_14B
    corpus_path: str = "data/midtrain/corpus.jsonl"
    output_dir: str = "runs/midtrain"
    general_replay_frac: float = 0.30
    learning_rate: float = 1e-5
    lr_scheduler_type: str = "cosine"
    num_train_epochs: float = 1.0
    warmup_ratio: float = 0.05
    max_seq_length: int = 8192
    bf16: bool = True
    gradient_checkpointing: bool = True
    use_lora: bool = False
    per_device_train_batch_size: int = 4
    gradient_accumulation_steps: int = 4
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0
    packing: bool = False
    logging_steps: int = 10
    save_steps: int = 200
    save_total_limit: int = 1
    seed: int = 0
    max_steps: int = -1


@dataclass
class MultiCapSFTConfig(SFTConfig):
    frac_kernel_repair_opt: float = 0.28
    frac_kernel_qa: float = 0.10
    frac_agentic_tooluse: float = 0.12
    frac_general_code: float = 0.13
    frac_math_reasoning: float = 0.10
    frac_general_chat: float = 0.27
    use_lora: bool = False
    num_train_epochs: float = 3.0


@dataclass
class SoupConfig:
    base_model_id: str = MODEL_14B
    kore_checkpoint: str = "runs/grpo"
    output_dir: str = "runs/soup"
    alphas: tuple = (0.7, 0.8, 0.9)
    epsilon: float = 0.005


# ---------------------------------------------------------------------- helpers
def detect_transformer_layer_cls(model_id: str) -> str:
    """Decoder-layer class name for a HF model id (kept for config compatibility)."""
    mid = (model_id or "").lower()
    if "llama" in mid:
        return "LlamaDecoderLayer"
    if "qwen3" in mid and "moe" in mid:
        return "Qwen3MoeDecoderLayer"
    if "qwen3" in mid:
        return "Qwen3DecoderLayer"
    if "qwen" in mid:
        return "Qwen2DecoderLayer"
    if "mistral" in mid:
        return "MistralDecoderLayer"
    return "Qwen3DecoderLayer"


def fsdp_enabled(config) -> bool:
    """Sharded full fine-tuning only when ``distributed`` and not LoRA."""
    return bool(getattr(config, "distributed", False)) and not bool(getattr(config, "use_lora", False))


def sharding_plan(config, world: int) -> dict:
    """Map the reference's FSDP / ZeRO knobs onto this framework's plan.

    Returns {"zero": 0|2|3, "offload": bool}. ``full_shard`` -> ZeRO-3
    (parameters sharded, gathered per unit); ``shard_grad_op`` or GRPO ->
    ZeRO-2; world 1 -> 0."""
    if world <= 1 or not fsdp_enabled(config):
        return {"zero": 0, "offload": False}
    s = (getattr(config, "fsdp", "") or "").lower()
    zero = 3 if "full_shard" in s else 2
    if isinstance(config, GRPOConfig):
        zero = 2
    return {"zero": zero, "offload": bool(getattr(config, "fsdp_cpu_offload", False))}


def parallel_kwargs(config, world: int) -> dict:
    """CausalLMTrainer arguments of this config: ZeRO-3 (full_shard) runs on
    NCCL collectives, ZeRO-2 on the configured data plane."""
    z = sharding_plan(config, world)["zero"]
    if z == 3:
        return {"zero_stage": 3, "comm": "nccl"}
    return {"zero_stage": 2, "comm": getattr(config, "comm", "nccl")}


def build_fsdp_kwargs(config) -> dict:
    """The reference's HF-Trainer FSDP kwargs for this config ({} when not
    distributed). Kept so tools that inspect them keep working; the engine
    itself consumes :func:`sharding_plan`."""
    if not fsdp_enabled(config):
        return {}
    layer_cls = (getattr(config, "fsdp_transformer_layer_cls", None)
                 or detect_transformer_layer_cls(getattr(config, "model_id", "")))
    s = getattr(config, "fsdp", "full_shard auto_wrap") or "full_shard auto_wrap"
    if getattr(config, "fsdp_cpu_offload", False) and "offload" not in s:
        s = f"{s} offload"
    cfg = {"transformer_layer_cls_to_wrap": [layer_cls], "backward_prefetch": "backward_pre",
           "forward_prefetch": True, "use_orig_params": True, "sync_module_states": True,
           "cpu_ram_efficient_loading": True, "limit_all_gathers": True,
           "state_dict_type": "FULL_STATE_DICT"}
    if getattr(config, "fsdp_cpu_offload", False):
        cfg["offload_params"] = True
    return {"fsdp": s, "fsdp_config": cfg}


def checkpoint_intact(path: str) -> bool:
    """Every safetensors file in ``path`` has a readable header and exactly the
    bytes its header declares (catches files truncated by a crash mid-save)."""
    import json as _json
    import struct
    for f in glob.glob(os.path.join(path, "*.safetensors")):
        try:
            size = os.path.getsize(f)
            with open(f, "rb") as fh:
                n = struct.unpack("<Q", fh.read(8))[0]
                if n <= 0 or 8 + n > size:
                    return False
                hdr = _json.loads(fh.read(n))
            end = max((v["data_offsets"][1] for k, v in hdr.items() if k != "__metadata__"), default=0)
            if 8 + n + end != size:
                return False
        except (OSError, ValueError, KeyError, struct.error):
            return False
    return True


def latest_checkpoint(output_dir) -> Optional[str]:
    """Newest intact ``checkpoint-<step>`` directory that has ``trainer_state.json``
    (a checkpoint left corrupt by a crash is skipped for the previous one)."""
    cands = [c for c in glob.glob(os.path.join(str(output_dir), "checkpoint-*")) if os.path.isdir(c)]

    def step(p):
        try:
            return int(os.path.basename(p).rsplit("-", 1)[1])
        except (ValueError, IndexError):
            return -1

    cands.sort(key=step)
    for c in reversed(cands):
        if os.path.exists(os.path.join(c, "trainer_state.json")) and checkpoint_intact(c):
            return c
    return None


def preferred_attn_impl() -> str:
    """The attention implementation the engine runs: the native tcgen05 kernel."""
    return "kore_tcgen05"


def grpo_distributed_enabled(config) -> bool:
    return fsdp_enabled(config)


def grpo_sharding_backend(config) -> str:
    """"none" outside distributed full-FT, else "fsdp" (the engine's sharding;
    "deepspeed" is accepted and mapped onto the same engine)."""
    if not grpo_distributed_enabled(config):
        return "none"
    want = (getattr(config, "sharding_backend", "auto") or "auto").lower()
    return "deepspeed" if want == "deepspeed" else "fsdp"


def build_deepspeed_config(config) -> dict:
    """ZeRO config dict equivalent of this config (for inspection / export)."""
    path = getattr(config, "ds_config", None)
    if path:
        with open(path) as f:
            return json.load(f)
    stage = int(getattr(config, "zero_stage", 3))
    zero = {"stage": stage, "overlap_comm": True, "contiguous_gradients": True,
            "reduce_bucket_size": "auto"}
    if stage == 3:
        zero.update({"stage3_gather_16bit_weights_on_model_save": True,
                     "stage3_param_persistence_threshold": "auto",
                     "stage3_prefetch_bucket_size": "auto",
                     "stage3_max_live_parameters": int(1e9),
                     "stage3_max_reuse_distance": int(1e9)})
    if getattr(config, "cpu_offload", False):
        zero["offload_param"] = {"device": "cpu", "pin_memory": True}
        zero["offload_optimizer"] = {"device": "cpu", "pin_memory": True}
    return {"train_micro_batch_size_per_gpu": 1, "gradient_accumulation_steps": 1,
            "gradient_clipping": float(getattr(config, "max_grad_norm", 1.0)),
            "bf16": {"enabled": bool(getattr(config, "bf16", True))}, "fp16": {"enabled": False},
            "zero_optimization": zero}


# ------------------------------------------------------------- dict -> config
def _build(cls, d: dict, extras=()):
    d = dict(d)
    lora = d.pop("lora", None)
    ext = {k: d.pop(k) for k in list(d) if k in extras}
    names = {f.name for f in fields(cls)}
    unknown = [k for k in d if k not in names]
    if unknown:
        raise TypeError(f"{cls.__name__}: unknown config keys {unknown}")
    cfg = cls(**d)
    if lora is not None and hasattr(cfg, "lora"):
        cfg.lora = LoRAConfig(**lora)
    for k, v in ext.items():
        if v is not None:
            setattr(cfg, k, v)
    return cfg


def sft_config_from_dict(d: dict):
    """(SFTConfig, dataset_path) from a JSON dict (nested ``lora`` allowed)."""
    cfg = _build(SFTConfig, d)
    return cfg, cfg.dataset_path


DPO_EXTRAS = ("loss_type", "loss_weights", "label_smoothing", "ld_alpha", "truncation_mode",
              "max_grad_norm")


def dpo_config_from_dict(d: dict) -> DPOConfig:
    """DPOConfig; the TRL-style loss knobs (``loss_type`` list for RPO/IPO,
    ``label_smoothing``, ``ld_alpha``, ``truncation_mode``, ``max_grad_norm``)
    are attached as attributes."""
    return _build(DPOConfig, d, extras=DPO_EXTRAS)


def grpo_config_from_dict(d: dict) -> GRPOConfig:
    """GRPOConfig; ``tasks`` (the campaign's task list) and a stale ``lora``
    block are dropped (GRPO is full fine-tuning)."""
    d = dict(d)
    d.pop("tasks", None)
    d.pop("lora", None)
    return _build(GRPOConfig, d)


def midtrain_config_from_dict(d: dict) -> MidTrainConfig:
    return _build(MidTrainConfig, d)


def config_to_dict(cfg) -> dict:
    return asdict(cfg)
