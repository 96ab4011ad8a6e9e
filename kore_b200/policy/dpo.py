"""Direct Preference Optimization on the explicit engine.

Each step takes chosen/rejected pairs, computes the frozen reference
model's sequence log-probs, then runs the policy with a two-phase head: the
micro-batch's response log-probs give the loss and the per-token
coefficients dL/dlogp_t, which the engine turns into gradients. Losses
(``loss_type`` may be a list, weighted by ``loss_weights``):

* ``sigmoid`` — DPO, with ``label_smoothing`` eps (cDPO):
  -(1-eps) log s(beta*h) - eps log s(-beta*h), h = (pi_c - ref_c) - (pi_r - ref_r)
* ``ipo`` — (h_mean - 1/(2 beta))^2 on token-mean log-probs
* ``sft`` — NLL of the chosen response (token mean); ["sigmoid", "sft"] = RPO
* ``ld_alpha`` (LD-DPO): tokens past the shorter response's length count
  with weight alpha in the sequence log-prob
* ``truncation_mode="keep_end"``: prompts are left-truncated to fit.

Behavioural parity: kore/policy/dpo.py:64-450 (TRL DPOTrainer knobs).
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path
from typing import List, Optional

import torch

from ..data.datasets import load_dpo_rows
from ..data.tokenizer import _enc, load_tokenizer, render_chat
from ..models.hf_io import load_pretrained_or_init
from ..obs import configure, get_logger
from ..parallel.dist import init_distributed
from ._loop import plan_steps, run_loop
from .configs import DPOConfig, dpo_config_from_dict

log = get_logger("policy.dpo")


def _softplus(x: float) -> float:
    return math.log1p(math.exp(-abs(x))) + max(x, 0.0)


def _sigmoid(x: float) -> float:
    return 1.0 / (1.0 + math.exp(-x)) if x >= 0 else math.exp(x) / (1.0 + math.exp(x))


def dpo_pair_loss(pc, pr, rc, rr, nc, nr, *, beta, loss_types, loss_weights, label_smoothing=0.0):
    """Loss of one pair and its derivatives w.r.t. the policy SUM log-probs
    (pc, pr). rc/rr: reference sums; nc/nr: response token counts."""
    loss, dc, dr = 0.0, 0.0, 0.0
    for lt, lw in zip(loss_types, loss_weights):
        if lt == "sigmoid":
            h = (pc - rc) - (pr - rr)
            z = beta * h
            eps = label_smoothing
            loss += lw * ((1 - eps) * _softplus(-z) + eps * _softplus(z))
            g = (-(1 - eps) * _sigmoid(-z) + eps * _sigmoid(z)) * beta
            dc += lw * g
            dr -= lw * g
        elif lt == "ipo":
            h = (pc / nc - rc / nc) - (pr / nr - rr / nr)
            t = h - 1.0 / (2.0 * beta)
            loss += lw * t * t
            dc += lw * 2 * t / nc
            dr -= lw * 2 * t / nr
        elif lt == "sft":
            loss += lw * (-pc / nc)
            dc += lw * (-1.0 / nc)
        else:
            raise ValueError(f"unknown DPO loss_type {lt!r}")
    return loss, dc, dr


def encode_pair(tok, row, max_len: int, max_prompt: int, keep_end: bool):
    p_ids, _ = render_chat(tok, row["prompt"], add_generation_prompt=True)
    if keep_end and len(p_ids) > max_prompt:
        p_ids = p_ids[-max_prompt:]
    out = []
    for key in ("chosen", "rejected"):
        body = "".join(m.get("content", "") for m in row[key] if m.get("role", "assistant") == "assistant")
        r_ids = _enc(tok, body) + _enc(tok, "<|im_end|>")
        ids = (p_ids + r_ids)[:max_len] if not keep_end else (p_ids + r_ids)[-max_len:]
        n_ctx = max(1, len(ids) - len(r_ids))
        out.append((ids, n_ctx))
    return out


class DPOTrainer:
    def __init__(self, config: DPOConfig, ctx, weights, ref_weights=None, total_steps: int = 1):
        from ..engine.qwen3_engine import Qwen3Engine
        from ..engine.trainer import CausalLMTrainer
        self.cfg = config
        self.ctx = ctx
        self.tr = CausalLMTrainer(weights.cfg, ctx, lr=config.learning_rate, weight_decay=config.weight_decay,
                                  max_grad_norm=float(getattr(config, "max_grad_norm", 1.0)),
                                  seed=config.seed, schedule=config.lr_scheduler_type,
                                  warmup_steps=int(config.warmup_ratio * total_steps), total_steps=total_steps,
                                  weights=weights, comm=config.comm)
        self.ref_placement = self._choose_placement(getattr(config, "ref_placement", "auto"))
        self.ref = Qwen3Engine(self._build_ref(ref_weights), allocate_grads=False)
        if self.ref_placement != "resident":
            self.ref.param_hook = self._ref_stream
        self.micro_pairs = max(1, int(getattr(config, "micro_pairs", 1)))
        lt = getattr(config, "loss_type", "sigmoid")
        self.loss_types = lt if isinstance(lt, list) else [lt]
        lw = getattr(config, "loss_weights", None)
        self.loss_weights = lw if lw else [1.0] * len(self.loss_types)
        if len(self.loss_weights) != len(self.loss_types):
            raise ValueError("loss_weights must match loss_type in length")
        self.ld_alpha = getattr(config, "ld_alpha", None)
        self.eps = float(getattr(config, "label_smoothing", 0.0) or 0.0)

    def _choose_placement(self, mode: str) -> str:
        """Where the frozen reference's decoder layers live: resident in HBM,
        streamed from pinned host memory, or sharded over ranks and
        all-gathered layer by layer (the reference sharded alongside the policy).
        ``auto``: sharded with several ranks; on one GPU streamed from host when a
        second resident copy of the weights would not leave room for activations."""
        if mode != "auto":
            return mode
        if self.ctx.world > 1:
            return "shard"
        w = self.tr.w
        if w.device.type != "cuda":
            return "resident"
        free, _ = torch.cuda.mem_get_info(w.device)
        need = sum(b.numel() * b.element_size() for b in w.bufs if b is not None)
        return "host" if free < need + 24e9 else "resident"

    def _build_ref(self, ref_weights):
        from ..engine.frozen_stream import FrozenLayerStream
        from ..models import Qwen3Weights
        if self.ref_placement == "resident":
            return ref_weights if ref_weights is not None else self.tr.w.clone()
        src = ref_weights if ref_weights is not None else self.tr.w
        ref = Qwen3Weights(src.cfg, device=src.device, dtype=src.dtype, allocate=False,
                           pad_multiple=src.pad_multiple, ep=src.ep)
        last = src.num_units - 1
        ref.bufs = [src.bufs[u].clone() if u in (0, last) else None for u in range(src.num_units)]
        self._ref_stream = FrozenLayerStream(ref, source=self.ref_placement, ctx=self.ctx, layers_from=src)
        self._ref_hook = self._ref_stream
        return ref

    def _park_ref(self):
        """One GPU with the reference streamed from host memory: once all its
        log-probs of the step are computed, its resident units (embedding and
        head) move to pinned host memory and its layer ring is freed for the
        policy update; ``step`` brings them back after the optimizer step.
        Returns the parked slots, or None when nothing is parked."""
        if self.ctx.world > 1 or self.ctx.device.type != "cuda" or self.ref_placement != "host":
            return None
        from ..engine.offload import HostStash, weight_slots
        if not hasattr(self, "_ref_stash"):
            self._ref_stash = HostStash()
        st = self._ref_stream
        st.free_ring()
        rw = self.ref.w
        slots = [(c, k) for c, k in weight_slots(rw) if not (c is rw.bufs and k in st.store)]
        self._ref_stash.park(slots)
        return slots

    def _batch(self, items):
        from ..engine.qwen3_engine import Batch
        seqs, masks = [], []
        for ids, n_ctx in items:
            seqs.append(torch.tensor(ids, dtype=torch.long))
            m = torch.zeros(len(ids), dtype=torch.bool)
            m[n_ctx:] = True
            masks.append(m)
        return Batch.from_sequences(seqs, masks, device=self.ctx.device)

    def _token_weights(self, b, items):
        """Per label-position weight (LD-DPO alpha beyond the shared length) and segment ids."""
        seg = torch.full((b.num_tokens,), -1, dtype=torch.long)
        wt = torch.zeros(b.num_tokens, dtype=torch.float32)
        off = 0
        for i, (ids, n_ctx) in enumerate(items):
            L = len(ids)
            seg[off + n_ctx - 1: off + L - 1] = i
            wt[off + n_ctx - 1: off + L - 1] = 1.0
            if self.ld_alpha is not None:
                pair = i // 2
                other = items[i ^ 1]
                shared = min(L - n_ctx, len(other[0]) - other[1])
                wt[off + n_ctx - 1 + shared: off + L - 1] = float(self.ld_alpha)
            off += L
        return seg.to(b.ids.device), wt.to(b.ids.device)

    def step(self, pairs: List[list]) -> float:
        """pairs: list of [(chosen_ids, n_ctx), (rejected_ids, n_ctx)]; one
        optimizer step over micro-batches of ``micro_pairs`` pairs (a pair's
        loss depends only on its own sums, so micro-batching is exact)."""
        cfg = self.cfg
        npairs_t = torch.tensor([float(len(pairs))], device=self.ctx.device)
        self.ctx.all_reduce(npairs_t)
        npairs_global = float(npairs_t.item())
        eng = self.tr.eng
        eng.zero_grad()
        total = 0.0
        starts = list(range(0, len(pairs), self.micro_pairs))
        batches = [self._batch([x for p in pairs[s0:s0 + self.micro_pairs] for x in p]) for s0 in starts]
        if getattr(self, "_ref_stream", None) is not None:
            # streamed / gathered reference: each layer moves once for the whole step
            ref_lps = [lp for lp, _ in self.ref.token_logprobs_many(batches)]
        else:
            ref_lps = [None] * len(batches)
        parked = self._park_ref() if ref_lps[0] is not None else None
        # one GPU: the second moments leave HBM for the middle micro-batches, which
        # then keep their layer contexts instead of recomputing (None elsewhere)
        shuttle = self.tr._moment_shuttle(len(batches), max(b.num_tokens for b in batches))
        for i, (s0, b, lp_pre) in enumerate(zip(starts, batches, ref_lps)):
            if shuttle is not None:
                shuttle.before(i)
            chunk = pairs[s0:s0 + self.micro_pairs]
            items = [x for p in chunk for x in p]
            seg, wt = self._token_weights(b, items)
            lp_ref = lp_pre if lp_pre is not None else self.ref.token_logprobs(b)[0]
            n = len(items)
            ref_sums = torch.zeros(n, dtype=torch.float64, device=lp_ref.device)
            ref_sums.index_add_(0, seg.clamp_min(0), torch.where(seg >= 0, (lp_ref * wt).double(),
                                                                 torch.zeros_like(lp_ref.double())))
            ref_s = ref_sums.tolist()
            counts = [max(1, len(ids) - c) for ids, c in items]

            def coef_fn(lp_full, seg=seg, wt=wt, n=n, ref_s=ref_s, counts=counts, np_=len(chunk)):
                sums = torch.zeros(n, dtype=torch.float64, device=lp_full.device)
                sums.index_add_(0, seg.clamp_min(0), torch.where(seg >= 0, (lp_full * wt).double(),
                                                                 torch.zeros_like(lp_full.double())))
                ps = sums.tolist()
                d = [0.0] * n
                loss = 0.0
                for k in range(np_):
                    c, r = 2 * k, 2 * k + 1
                    l, dc, dr = dpo_pair_loss(ps[c], ps[r], ref_s[c], ref_s[r], counts[c], counts[r],
                                              beta=cfg.beta, loss_types=self.loss_types,
                                              loss_weights=self.loss_weights, label_smoothing=self.eps)
                    loss += l / npairs_global
                    d[c] = dc / npairs_global
                    d[r] = dr / npairs_global
                dv = torch.tensor(d, dtype=torch.float32, device=lp_full.device)
                coef = torch.where(seg >= 0, dv[seg.clamp_min(0)] * wt, torch.zeros_like(lp_full))
                return coef, loss

            out = eng.forward_backward(b, coef_fn=coef_fn)
            total += float(out["loss"])
        if shuttle is not None:
            shuttle.finish()
        self.tr.opt.step()
        if parked is not None:
            self._ref_stash.restore(parked, self.ctx.device)
        loss = torch.tensor([total], device=self.ctx.device)
        self.ctx.all_reduce(loss)
        return float(loss.item())


def train(config: DPOConfig, *, model_cfg=None, tokenizer=None, weights=None, ref_weights=None) -> dict:
    ctx = init_distributed()
    configure(config.output_dir)
    tok = tokenizer or load_tokenizer(config.model_id)
    rows = load_dpo_rows(config.dataset_path)
    keep_end = getattr(config, "truncation_mode", "keep_end") == "keep_end"
    pairs = [encode_pair(tok, r, config.max_length, config.max_prompt_length, keep_end) for r in rows]
    w = weights or load_pretrained_or_init(config.model_id, ctx, model_cfg=model_cfg, bf16=config.bf16,
                                           seed=config.seed)
    if ref_weights is None and config.ref_model_id and config.ref_model_id != config.model_id:
        ref_weights = load_pretrained_or_init(config.ref_model_id, ctx, model_cfg=model_cfg, bf16=config.bf16,
                                              seed=config.seed)
    total = plan_steps(len(pairs), ctx.world, config.per_device_train_batch_size,
                       config.gradient_accumulation_steps, config.num_train_epochs, config.max_steps)
    dt = DPOTrainer(config, ctx, w, ref_weights, total_steps=total)
    return run_loop("dpo", pairs, dt.step, ctx=ctx, trainer=dt.tr, tokenizer=tok, output_dir=config.output_dir,
                    per_device=config.per_device_train_batch_size, accum=config.gradient_accumulation_steps,
                    epochs=config.num_train_epochs, max_steps=config.max_steps,
                    logging_steps=config.logging_steps, save_steps=config.save_steps, seed=config.seed)


def _main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print("usage: python -m kore_b200.policy.dpo <config.json>", file=sys.stderr)
        return 2
    raw = json.loads(Path(argv[0]).read_text())
    raw.setdefault("distributed", True)
    cfg = dpo_config_from_dict(raw)
    print(f"[dpo] -> {train(cfg)['output_dir']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
