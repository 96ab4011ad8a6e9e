"""Qwen3 dense / Qwen3-MoE weights held in flat per-unit buffers.

A model is a list of *units*: unit 0 is the token embedding, units 1..L are
decoder layers, unit L+1 is the head (final RMSNorm + lm_head). Each unit's
parameters live in ONE contiguous bf16 buffer with named, 256-byte-aligned
segments. That single layout serves every consumer:

* the GEMMs read fused views (q|k|v stacked as one [(Hq+2Hkv)*D, H] weight,
  gate|up stacked as one [2F, H] weight) straight out of the buffer;
* FSDP shards, all-gathers and reduce-scatters whole units;
* the fused AdamW kernel updates a unit with one launch;
* HF safetensors load/save maps HF key names onto segment slices, so
  checkpoints use exactly HF's Qwen3 key names and shapes.

Reference parity: the reference holds these weights inside HF
``Qwen3ForCausalLM`` (kore/policy/grpo.py:2017-2018) and saves them with
``save_pretrained`` (kore/policy/grpo.py:2320-2331).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from .config import Qwen3Config

ALIGN = 128  # elements (256 B for bf16): keeps every segment TMA-aligned


def _round_up(x: int, a: int = ALIGN) -> int:
    return (x + a - 1) // a * a


@dataclass
class Segment:
    name: str
    shape: Tuple[int, ...]
    offset: int
    init: str  # "normal" | "ones" | "zeros"

    @property
    def numel(self) -> int:
        return int(math.prod(self.shape))


class UnitLayout:
    """Named segments of one flat buffer."""

    def __init__(self, kind: str, segs: List[Tuple[str, Tuple[int, ...], str]]):
        self.kind = kind
        self.segments: Dict[str, Segment] = {}
        off = 0
        for name, shape, init in segs:
            self.segments[name] = Segment(name, tuple(shape), off, init)
            off = _round_up(off + int(math.prod(shape)))
        self.numel = off

    def views(self, buf: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {n: buf[s.offset: s.offset + s.numel].view(s.shape) for n, s in self.segments.items()}


def layer_layout(cfg: Qwen3Config, i: int) -> UnitLayout:
    H, D = cfg.hidden_size, cfg.head_dim
    segs = [
        ("ln1", (H,), "ones"),
        ("qkv", (cfg.q_dim + 2 * cfg.kv_dim, H), "normal"),
        ("q_norm", (D,), "ones"),
        ("k_norm", (D,), "ones"),
        ("o", (H, cfg.q_dim), "normal"),
        ("ln2", (H,), "ones"),
    ]
    if cfg.layer_is_moe(i):
        E, I = cfg.num_experts, cfg.moe_intermediate_size
        segs += [("router", (E, H), "normal"),
                 ("experts_gate_up", (E, 2 * I, H), "normal"),
                 ("experts_down", (E, H, I), "normal")]
        return UnitLayout("moe_layer", segs)
    F = cfg.intermediate_size
    segs += [("gate_up", (2 * F, H), "normal"), ("down", (H, F), "normal")]
    return UnitLayout("layer", segs)


def unit_layouts(cfg: Qwen3Config) -> List[UnitLayout]:
    H, V = cfg.hidden_size, cfg.vocab_size
    units = [UnitLayout("embed", [("embed", (V, H), "normal")])]
    units += [layer_layout(cfg, i) for i in range(cfg.num_hidden_layers)]
    head = [("norm", (H,), "ones")]
    if not cfg.tie_word_embeddings:
        head.append(("lm_head", (V, H), "normal"))
    units.append(UnitLayout("head", head))
    return units


def hf_names(cfg: Qwen3Config, unit: int, layout: UnitLayout):
    """Yield (hf_key, segment_name, row_slice or None, expert index or None)."""
    L = cfg.num_hidden_layers
    if unit == 0:
        yield "model.embed_tokens.weight", "embed", None, None
        return
    if unit == L + 1:
        yield "model.norm.weight", "norm", None, None
        if not cfg.tie_word_embeddings:
            yield "lm_head.weight", "lm_head", None, None
        return
    i = unit - 1
    p = f"model.layers.{i}."
    qd, kd = cfg.q_dim, cfg.kv_dim
    yield p + "input_layernorm.weight", "ln1", None, None
    yield p + "self_attn.q_proj.weight", "qkv", (0, qd), None
    yield p + "self_attn.k_proj.weight", "qkv", (qd, qd + kd), None
    yield p + "self_attn.v_proj.weight", "qkv", (qd + kd, qd + 2 * kd), None
    yield p + "self_attn.q_norm.weight", "q_norm", None, None
    yield p + "self_attn.k_norm.weight", "k_norm", None, None
    yield p + "self_attn.o_proj.weight", "o", None, None
    yield p + "post_attention_layernorm.weight", "ln2", None, None
    if layout.kind == "moe_layer":
        I = cfg.moe_intermediate_size
        yield p + "mlp.gate.weight", "router", None, None
        for e in range(cfg.num_experts):
            q = p + f"mlp.experts.{e}."
            yield q + "gate_proj.weight", "experts_gate_up", (0, I), e
            yield q + "up_proj.weight", "experts_gate_up", (I, 2 * I), e
            yield q + "down_proj.weight", "experts_down", None, e
    else:
        F = cfg.intermediate_size
        yield p + "mlp.gate_proj.weight", "gate_up", (0, F), None
        yield p + "mlp.up_proj.weight", "gate_up", (F, 2 * F), None
        yield p + "mlp.down_proj.weight", "down", None, None


def _dtype(name: str) -> torch.dtype:
    return {"bfloat16": torch.bfloat16, "float32": torch.float32,
            "float16": torch.float16}.get(name, torch.bfloat16)


class Qwen3Weights:
    """All parameters of a Qwen3(-MoE) causal LM as flat per-unit buffers.

    ``units`` selects which units this object materialises (all by default);
    FSDP uses full buffers for gathering and keeps only shards resident.
    """

    def __init__(self, cfg: Qwen3Config, device="cpu", dtype: Optional[torch.dtype] = None,
                 init: bool = True, seed: int = 0, std: float = 0.02,
                 allocate: bool = True, pad_multiple: int = ALIGN, alloc=None):
        self.cfg = cfg
        self.dtype = dtype or _dtype(cfg.torch_dtype)
        self.device = torch.device(device)
        self.layouts = unit_layouts(cfg)
        # buffers are padded so that data-parallel shards divide them evenly
        self.pad_multiple = max(ALIGN, int(pad_multiple))
        self.bufs: List[Optional[torch.Tensor]] = [None] * len(self.layouts)
        if allocate:
            for u, lay in enumerate(self.layouts):
                # ``alloc(numel, dtype)`` lets callers place the buffers (e.g. in
                # the symmetric peer-memory heap of the fused collectives)
                self.bufs[u] = (alloc(self.padded_numel(u), self.dtype) if alloc is not None else
                                torch.empty(self.padded_numel(u), dtype=self.dtype, device=self.device))
            if init:
                self.init_random(seed, std)

    def padded_numel(self, u: int) -> int:
        return _round_up(self.layouts[u].numel, self.pad_multiple)

    # ------------------------------------------------------------------ views
    def views(self, u: int) -> Dict[str, torch.Tensor]:
        return self.layouts[u].views(self.bufs[u])

    @property
    def num_units(self) -> int:
        return len(self.layouts)

    def numel(self) -> int:
        return sum(l.numel for l in self.layouts)

    def lm_head_weight(self) -> torch.Tensor:
        if self.cfg.tie_word_embeddings:
            return self.views(0)["embed"]
        return self.views(self.num_units - 1)["lm_head"]

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float = 0.02) -> None:
        """Random init like HF's ``_init_weights``: N(0, std) for matrices,
        ones for norm weights; segment padding is zeroed. Generated on the
        buffer's device (seeded per unit, so it is reproducible)."""
        for u, lay in enumerate(self.layouts):
            buf = self.bufs[u]
            buf.zero_()
            g = torch.Generator(device=buf.device)
            g.manual_seed(seed * 1000003 + u)
            for name, v in lay.views(buf).items():
                init = lay.segments[name].init
                if init == "ones":
                    v.fill_(1.0)
                elif init == "normal":
                    if v.dtype in (torch.float32, torch.float64):
                        v.normal_(0.0, std, generator=g)
                    else:
                        t = torch.empty(v.shape, dtype=torch.float32, device=v.device)
                        # generate in row blocks to bound the fp32 temporary
                        flat = v.view(v.shape[0], -1) if v.dim() > 1 else v.view(1, -1)
                        step = max(1, (1 << 26) // max(1, flat.shape[1]))
                        tf = t.view(flat.shape)
                        for r in range(0, flat.shape[0], step):
                            tf[r: r + step].normal_(0.0, std, generator=g)
                            flat[r: r + step].copy_(tf[r: r + step])
                        del t

    # ------------------------------------------------------------------ HF io
    def hf_state_dict(self) -> Dict[str, torch.Tensor]:
        """HF Qwen3 key -> tensor view (no copies)."""
        out = {}
        for u, lay in enumerate(self.layouts):
            if self.bufs[u] is None:
                continue
            vs = lay.views(self.bufs[u])
            for key, seg, rows, expert in hf_names(self.cfg, u, lay):
                t = vs[seg]
                if expert is not None:
                    t = t[expert]
                if rows is not None:
                    t = t[rows[0]: rows[1]]
                out[key] = t
        return out

    @torch.no_grad()
    def load_hf_state_dict(self, sd: Dict[str, torch.Tensor], strict: bool = True) -> List[str]:
        mine = self.hf_state_dict()
        missing = []
        for k, dst in mine.items():
            if k not in sd:
                if k == "lm_head.weight" and self.cfg.tie_word_embeddings:
                    continue
                missing.append(k)
                continue
            src = sd[k]
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"shape mismatch for {k}: {tuple(src.shape)} vs {tuple(dst.shape)}")
            dst.copy_(src.to(dst.dtype))
        if strict and missing:
            raise KeyError(f"missing keys: {missing[:8]}{'...' if len(missing) > 8 else ''}")
        return missing

    def to(self, device=None, dtype=None) -> "Qwen3Weights":
        w = Qwen3Weights(self.cfg, device or self.device, dtype or self.dtype, allocate=False,
                         pad_multiple=self.pad_multiple)
        w.bufs = [b.to(device=w.device, dtype=w.dtype) if b is not None else None for b in self.bufs]
        return w

    def clone(self) -> "Qwen3Weights":
        w = Qwen3Weights(self.cfg, self.device, self.dtype, allocate=False,
                         pad_multiple=self.pad_multiple)
        w.bufs = [b.clone() if b is not None else None for b in self.bufs]
        return w
