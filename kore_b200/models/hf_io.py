"""HF-format checkpoints: safetensors shards with Qwen3 key names.

``save_pretrained`` writes ``config.json``, ``model-XXXXX-of-YYYYY.safetensors``
shards (<= 5 GB each) plus ``model.safetensors.index.json``, the tokenizer
(when it can save itself), and optionally ``trainer_state.json`` /
``optimizer.pt`` for mid-stage resume; ``keep_last`` prunes older
``checkpoint-*`` siblings. ``load_weights`` reads single-file or sharded
checkpoints straight into the flat unit buffers. The on-disk layout and key
names are exactly those ``transformers`` uses for Qwen3 / Qwen3-MoE, so
checkpoints round-trip with HF (reference: save_pretrained with a gathered
FULL_STATE_DICT, kore/policy/grpo.py:2320-2331, configs.py:640-647).
"""
from __future__ import annotations

import glob
import json
import os
import shutil
from typing import Dict, Optional

import torch

from ..obs import get_logger
from .config import PRESETS, Qwen3Config, qwen3_14b
from .qwen3 import Qwen3Weights

log = get_logger("models.hf_io")
SHARD_BYTES = 5 << 30


def save_pretrained(w: Qwen3Weights, out_dir: str, tokenizer=None, *, keep_last: int = 0,
                    trainer_state: Optional[dict] = None, optimizer_state: Optional[dict] = None) -> str:
    from safetensors.torch import save_file
    os.makedirs(out_dir, exist_ok=True)
    cfg = w.cfg.to_dict()
    cfg["torch_dtype"] = {torch.bfloat16: "bfloat16", torch.float32: "float32",
                          torch.float16: "float16"}.get(w.dtype, "bfloat16")
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    sd = w.hf_state_dict()
    shards, cur, size = [], {}, 0
    for k in sd:
        t = sd[k]
        nb = t.numel() * t.element_size()
        if cur and size + nb > SHARD_BYTES:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t
        size += nb
    if cur:
        shards.append(cur)
    n = len(shards)
    index = {"metadata": {"total_size": sum(t.numel() * t.element_size() for t in sd.values())},
             "weight_map": {}}
    for i, sh in enumerate(shards):
        name = "model.safetensors" if n == 1 else f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_file({k: v.detach().contiguous().cpu() for k, v in sh.items()}, os.path.join(out_dir, name),
                  metadata={"format": "pt"})
        for k in sh:
            index["weight_map"][k] = name
    if n > 1:
        with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
            json.dump(index, f, indent=2)
    if tokenizer is not None and hasattr(tokenizer, "save_pretrained"):
        try:
            tokenizer.save_pretrained(out_dir)
        except Exception as e:  # noqa: BLE001 - tokenizer save is best-effort
            log.warn("tokenizer save failed", err=str(e))
    if trainer_state is not None:
        with open(os.path.join(out_dir, "trainer_state.json"), "w") as f:
            json.dump(trainer_state, f, indent=2)
    if optimizer_state is not None:
        torch.save(optimizer_state, os.path.join(out_dir, "optimizer.pt"))
    if keep_last:
        parent = os.path.dirname(os.path.abspath(out_dir))
        ck = sorted(glob.glob(os.path.join(parent, "checkpoint-*")),
                    key=lambda p: int(p.rsplit("-", 1)[-1]) if p.rsplit("-", 1)[-1].isdigit() else -1)
        for old in ck[:-keep_last]:
            if os.path.abspath(old) != os.path.abspath(out_dir):
                shutil.rmtree(old, ignore_errors=True)
    return out_dir


def _checkpoint_files(path: str):
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            return sorted(set(json.load(f)["weight_map"].values()))
    files = sorted(os.path.basename(p) for p in glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no safetensors in {path}")
    return files


@torch.no_grad()
def load_weights(w: Qwen3Weights, path: str, strict: bool = True) -> None:
    from safetensors import safe_open
    mine = w.hf_state_dict()
    seen = set()
    dev = str(w.device)
    for fn in _checkpoint_files(path):
        with safe_open(os.path.join(path, fn), framework="pt", device=dev if w.device.type == "cuda" else "cpu") as f:
            for k in f.keys():
                if k in mine:
                    t = f.get_tensor(k)
                    if tuple(t.shape) != tuple(mine[k].shape):
                        raise ValueError(f"{k}: {tuple(t.shape)} vs {tuple(mine[k].shape)}")
                    mine[k].copy_(t.to(mine[k].dtype))
                    seen.add(k)
    missing = [k for k in mine if k not in seen and not (k == "lm_head.weight" and w.cfg.tie_word_embeddings)]
    if strict and missing:
        raise KeyError(f"checkpoint {path} misses {len(missing)} tensors, e.g. {missing[:4]}")


def from_pretrained(path: str, device="cpu", dtype=None, pad_multiple: int = 128) -> Qwen3Weights:
    cfg = Qwen3Config.from_pretrained(path)
    w = Qwen3Weights(cfg, device=device, dtype=dtype, init=False, pad_multiple=pad_multiple)
    for b in w.bufs:
        b.zero_()
    load_weights(w, path)
    return w


def resolve_config(model_id: Optional[str]) -> Qwen3Config:
    if model_id and os.path.exists(os.path.join(model_id, "config.json")):
        return Qwen3Config.from_pretrained(model_id)
    key = (model_id or "").lower().split("/")[-1]
    for name, fn in PRESETS.items():
        if name == key or name.replace("qwen3-", "") in key:
            return fn()
    if "30b-a3b" in key or "coder-30b" in key:
        return PRESETS["qwen3-coder-30b-a3b"]()
    return qwen3_14b()


def load_pretrained_or_init(model_id: Optional[str], ctx, *, model_cfg: Optional[Qwen3Config] = None,
                            bf16: bool = True, seed: int = 0) -> Qwen3Weights:
    """Local HF checkpoint when ``model_id`` is a directory with weights, else
    a random init of the architecture it names (there is no network)."""
    dev = ctx.device
    dtype = torch.bfloat16 if (bf16 and dev.type == "cuda") else torch.float32
    pad = 128 * max(1, ctx.world)
    if model_cfg is None and model_id and os.path.isdir(model_id) and glob.glob(os.path.join(model_id, "*.safetensors")):
        cfg = Qwen3Config.from_pretrained(model_id)
        w = Qwen3Weights(cfg, device=dev, dtype=dtype, init=False, pad_multiple=pad)
        for b in w.bufs:
            b.zero_()
        load_weights(w, model_id)
        return w
    cfg = model_cfg or resolve_config(model_id)
    log.info("random init (no local checkpoint)", model_id=str(model_id), layers=cfg.num_hidden_layers)
    return Qwen3Weights(cfg, device=dev, dtype=dtype, seed=seed, pad_multiple=pad)
