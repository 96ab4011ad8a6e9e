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


def expert_range(cfg: Qwen3Config, ep: Optional[Tuple[int, int]]) -> Tuple[int, int]:
    """Global expert ids [lo, hi) owned by rank ``ep[0]`` of ``ep[1]`` (all when no EP)."""
    if not ep or ep[1] <= 1:
        return 0, cfg.num_experts
    r, w = ep
    if cfg.num_experts % w:
        raise ValueError("num_experts must be divisible by the expert-parallel size")
    n = cfg.num_experts // w
    return r * n, (r + 1) * n


def expert_layout(cfg: Qwen3Config, n_local: int) -> UnitLayout:
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    return UnitLayout("experts", [("experts_gate_up", (n_local, 2 * I, H), "normal"),
                                  ("experts_down", (n_local, H, I), "normal")])


def layer_layout(cfg: Qwen3Config, i: int, with_experts: bool = True) -> UnitLayout:
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
        segs += [("router", (E, H), "normal")]
        if with_experts:
            segs += [("experts_gate_up", (E, 2 * I, H), "normal"),
                     ("experts_down", (E, H, I), "normal")]
        return UnitLayout("moe_layer", segs)
    F = cfg.intermediate_size
    segs += [("gate_up", (2 * F, H), "normal"), ("down", (H, F), "normal")]
    return UnitLayout("layer", segs)


def unit_layouts(cfg: Qwen3Config, with_experts: bool = True) -> List[UnitLayout]:
    H, V = cfg.hidden_size, cfg.vocab_size
    units = [UnitLayout("embed", [("embed", (V, H), "normal")])]
    units += [layer_layout(cfg, i, with_experts) for i in range(cfg.num_hidden_layers)]
    head = [("norm", (H,), "ones")]
    if not cfg.tie_word_embeddings:
        head.append(("lm_head", (V, H), "normal"))
    units.append(UnitLayout("head", head))
    return units


def hf_names(cfg: Qwen3Config, unit: int, layout: UnitLayout, expert_base: int = 0):
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
    if layout.kind == "experts":
        yield from _expert_names(cfg, p, layout, expert_base)
        return
    yield p + "input_layernorm.weight", "ln1", None, None
    yield p + "self_attn.q_proj.weight", "qkv", (0, qd), None
    yield p + "self_attn.k_proj.weight", "qkv", (qd, qd + kd), None
    yield p + "self_attn.v_proj.weight", "qkv", (qd + kd, qd + 2 * kd), None
    yield p + "self_attn.q_norm.weight", "q_norm", None, None
    yield p + "self_attn.k_norm.weight", "k_norm", None, None
    yield p + "self_attn.o_proj.weight", "o", None, None
    yield p + "post_attention_layernorm.weight", "ln2", None, None
    if layout.kind == "moe_layer":
        yield p + "mlp.gate.weight", "router", None, None
        yield from _expert_names(cfg, p, layout, expert_base)
    else:
        F = cfg.intermediate_size
        yield p + "mlp.gate_proj.weight", "gate_up", (0, F), None
        yield p + "mlp.up_proj.weight", "gate_up", (F, 2 * F), None
        yield p + "mlp.down_proj.weight", "down", None, None


def _expert_names(cfg, p, layout, expert_base):
    if "experts_gate_up" not in layout.segments:
        return
    I = cfg.moe_intermediate_size
    for e in range(layout.segments["experts_gate_up"].shape[0]):
        q = p + f"mlp.experts.{expert_base + e}."
        yield q + "gate_proj.weight", "experts_gate_up", (0, I), e
        yield q + "up_proj.weight", "experts_gate_up", (I, 2 * I), e
        yield q + "down_proj.weight", "experts_down", None, e


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
                 allocate: bool = True, pad_multiple: int = ALIGN, alloc=None,
                 ep: Optional[Tuple[int, int]] = None):
        self.cfg = cfg
        self.dtype = dtype or _dtype(cfg.torch_dtype)
        self.device = torch.device(device)
        # expert parallelism: MoE expert weights live in separate per-rank
        # buffers (only this rank's experts); everything else is replicated
        self.ep = ep if (ep and ep[1] > 1 and cfg.is_moe) else None
        self.expert_lo, self.expert_hi = expert_range(cfg, self.ep)
        self.layouts = unit_layouts(cfg, with_experts=self.ep is None)
        self.expert_layouts: Dict[int, UnitLayout] = {}
        self.expert_bufs: Dict[int, torch.Tensor] = {}
        if self.ep is not None:
            for i in range(cfg.num_hidden_layers):
                if cfg.layer_is_moe(i):
                    self.expert_layouts[i + 1] = expert_layout(cfg, self.expert_hi - self.expert_lo)
        # buffers are padded so that data-parallel shards divide them evenly
        self.pad_multiple = max(ALIGN, int(pad_multiple))
        self.bufs: List[Optional[torch.Tensor]] = [None] * len(self.layouts)
        if allocate:
            for u, lay in enumerate(self.layouts):
                # ``alloc(numel, dtype)`` lets callers place the buffers (e.g. in
                # the symmetric peer-memory heap of the fused collectives)
                self.bufs[u] = (alloc(self.padded_numel(u), self.dtype) if alloc is not None else
                                torch.empty(self.padded_numel(u), dtype=self.dtype, device=self.device))
            for u, lay in self.expert_layouts.items():
                self.expert_bufs[u] = torch.empty(lay.numel, dtype=self.dtype, device=self.device)
            if init:
                self.init_random(seed, std)

    def padded_numel(self, u: int) -> int:
        return _round_up(self.layouts[u].numel, self.pad_multiple)

    # ------------------------------------------------------------------ views
    def views(self, u: int) -> Dict[str, torch.Tensor]:
        v = self.layouts[u].views(self.bufs[u])
        if u in self.expert_bufs:
            v.update(self.expert_layouts[u].views(self.expert_bufs[u]))
        return v

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
        items = [(u, lay, self.bufs[u]) for u, lay in enumerate(self.layouts)]
        items += [(1000 + u, lay, self.expert_bufs[u]) for u, lay in self.expert_layouts.items()]
        for u, lay, buf in items:
            buf.zero_()
            g = torch.Generator(device=buf.device)
            g.manual_seed(seed * 1000003 + u + (7919 * self.expert_lo if u >= 1000 else 0))
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
            pairs = [(lay, vs, 0)]
            if u in self.expert_bufs:
                el = self.expert_layouts[u]
                pairs.append((el, el.views(self.expert_bufs[u]), self.expert_lo))
            for lay_, vs_, base in pairs:
                self._collect(out, u, lay_, vs_, base)
        return out

    def _collect(self, out, u, lay, vs, base):
        for key, seg, rows, expert in hf_names(self.cfg, u, lay, base):
            t = vs[seg]
            if expert is not None:
                t = t[expert]
            if rows is not None:
                t = t[rows[0]: rows[1]]
            out[key] = t

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
                         pad_multiple=self.pad_multiple, ep=self.ep)
        w.bufs = [b.to(device=w.device, dtype=w.dtype) if b is not None else None for b in self.bufs]
        w.expert_bufs = {u: b.to(device=w.device, dtype=w.dtype) for u, b in self.expert_bufs.items()}
        return w

    def clone(self) -> "Qwen3Weights":
        w = Qwen3Weights(self.cfg, self.device, self.dtype, allocate=False,
                         pad_multiple=self.pad_multiple, ep=self.ep)
        w.bufs = [b.clone() if b is not None else None for b in self.bufs]
        w.expert_bufs = {u: b.clone() for u, b in self.expert_bufs.items()}
        return w
