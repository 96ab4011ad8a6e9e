"""Causal-LM training step (SFT / midtrain) over one or more GPUs.

``CausalLMTrainer.train_step(ids, loss_mask)`` is the user-facing call: it
takes a host [B, S] token block (pinned memory is used when given), copies it
to the device, runs ``micro_batch_size``-sequence micro-batches through the
explicit engine with gradient accumulation, applies AdamW (sharded over
ranks when world > 1) and returns the global mean token loss as a float.
``train_step_device`` is the same step on device-resident inputs returning a
device scalar (no host sync).

The loss is the global token mean over every rank's labelled tokens
(reference: kore/policy/grpo.py:613-701 global token-mean; HF Trainer mean CE
for SFT, kore/policy/sft.py:346-399).
"""
from __future__ import annotations

from typing import Optional

import torch

from ..models import Qwen3Config, Qwen3Weights
from ..parallel.dist import DistContext, get_context
from .optimizer import AdamW
from .qwen3_engine import Batch, Qwen3Engine


def pick_master_mode(cfg: Qwen3Config, world: int, device: torch.device) -> str:
    """fp32 master when it fits, else stochastic-rounded bf16 params."""
    if device.type != "cuda":
        return "fp32"
    P = cfg.num_params()
    total = torch.cuda.get_device_properties(device).total_memory
    # bf16 params + bf16 grads + (m, v, master) sharded
    need_fp32 = 2 * P + 2 * P + 12 * P / world
    return "fp32" if need_fp32 < 0.86 * total else "none"


class CausalLMTrainer:
    def __init__(self, cfg: Qwen3Config, ctx: Optional[DistContext] = None, *, lr: float = 1e-5,
                 betas=(0.9, 0.95), weight_decay: float = 0.0, max_grad_norm: float = 1.0,
                 master: str = "auto", dtype: torch.dtype = torch.bfloat16, seed: int = 0,
                 micro_batch_size: int = 1, logits_chunk: int = 4096, schedule: str = "constant",
                 warmup_steps: int = 0, total_steps: int = 1, comm: str = "nccl",
                 weights: Optional[Qwen3Weights] = None, micro_tokens_hint: int = 8192,
                 ep_capacity: float = 2.0, zero_stage: int = 2, recompute: str = "auto",
                 activation_reserve_gb: float = 12.0, moment_offload: str = "auto", ep_dispatch: str = "push"):
        self.ctx = ctx or get_context()
        self.cfg = cfg
        dev = self.ctx.device
        self.heap = None
        grad_alloc = None
        ep = (self.ctx.rank, self.ctx.world) if (cfg.is_moe and self.ctx.world > 1) else None
        fused = comm == "fused" and self.ctx.world > 1 and dev.type == "cuda"
        self.zero_stage = zero_stage if self.ctx.world > 1 else 0
        gather_ce = fused and self.zero_stage == 3     # ZeRO-3: layer gathers on the copy engines
        if gather_ce:
            fused = False
        nvls = comm == "nvls" and self.ctx.world > 1 and dev.type == "cuda"
        if nvls and (self.zero_stage != 2 or cfg.is_moe):
            raise ValueError("comm='nvls' runs the dense ZeRO-2 step")
        self.nvls = None
        if fused or nvls:
            from ..parallel.symmetric import SymmetricHeap
            per = 128 * self.ctx.world
            from ..models.qwen3 import unit_layouts, _round_up
            tot = sum(_round_up(l.numel, per) for l in unit_layouts(cfg))
            n_units = len(unit_layouts(cfg))
            if nvls:
                from ..parallel.nvls import NVLSBuffers
                pbuf = NVLSBuffers(self.ctx, tot + 128 * n_units, dtype)
                gbuf = NVLSBuffers(self.ctx, tot + 128 * n_units, dtype)
                self.nvls = (pbuf, gbuf)
                self.heap = SymmetricHeap(self.ctx, 1 << 16)          # barrier / scalar signal pads only
                alloc = lambda n, dt: pbuf.alloc(n, dt)
                grad_alloc = lambda n, dt: gbuf.alloc(n, dt)
            else:
                self.heap = SymmetricHeap(self.ctx, 2 * tot * 2 + 256 * 4 * n_units)
                alloc = lambda n, dt: self.heap.alloc(n, dt)[1]
                grad_alloc = alloc
            if weights is None:
                weights = Qwen3Weights(cfg, device=dev, dtype=dtype, seed=seed, pad_multiple=per,
                                       alloc=alloc, ep=ep)
            else:  # move existing weights into the heap
                nw = Qwen3Weights(cfg, device=dev, dtype=weights.dtype, init=False, pad_multiple=per,
                                  alloc=alloc, ep=weights.ep)
                for a, b in zip(nw.bufs, weights.bufs):
                    a[: b.numel()].copy_(b[: a.numel()])
                for u, b in weights.expert_bufs.items():
                    nw.expert_bufs[u].copy_(b)
                # ownership moves into the heap: release the source buffers now
                # (the caller may still hold the old object)
                weights.bufs = [None] * len(weights.bufs)
                weights.expert_bufs = {}
                torch.cuda.empty_cache()
                weights = nw
        self.w = weights or Qwen3Weights(cfg, device=dev, dtype=dtype, seed=seed,
                                         pad_multiple=128 * max(1, self.ctx.world), ep=ep)
        self.eng = Qwen3Engine(self.w, logits_chunk=logits_chunk, grad_alloc=grad_alloc)
        if self.w.ep is not None:
            from ..parallel.ep import ExpertParallel, FusedExpertParallel
            if fused:
                from ..parallel.symmetric import SymmetricHeap
                cap = int(ep_capacity * micro_tokens_hint * cfg.num_experts_per_tok)
                ehp = SymmetricHeap(self.ctx, FusedExpertParallel.heap_bytes(cfg, cap, ep_dispatch) + (1 << 20))
                self.eng.ep = FusedExpertParallel(self.ctx, cfg, self.w.expert_lo, self.w.expert_hi, ehp, cap,
                                                  dispatch=ep_dispatch)
            else:
                self.eng.ep = ExpertParallel(self.ctx, cfg, self.w.expert_lo, self.w.expert_hi)
        if master == "auto":
            master = pick_master_mode(cfg, self.ctx.world, dev)
        self.master_mode = master
        self.mbs = micro_batch_size
        if nvls:
            from ..parallel.nvls import NVLSShardedAdamW
            self.opt = NVLSShardedAdamW(self.w, self.eng, self.ctx, self.nvls[0], self.nvls[1], self.heap, lr=lr,
                                        betas=betas, weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                                        master=master, schedule=schedule, warmup_steps=warmup_steps,
                                        total_steps=total_steps, seed=seed)
        elif fused:
            from ..parallel.zero import FusedShardedAdamW
            self.opt = FusedShardedAdamW(self.w, self.eng, self.ctx, self.heap, lr=lr, betas=betas,
                                         weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                                         master=master, schedule=schedule, warmup_steps=warmup_steps,
                                         total_steps=total_steps, seed=seed)
        elif self.zero_stage == 3:
            from ..parallel.fsdp import FullShard, FullShardAdamW
            self.fs = FullShard(self.w, self.eng, self.ctx, peer_gather=gather_ce)
            self.eng.param_hook = self.fs
            self.opt = FullShardAdamW(self.w, self.eng, self.ctx, self.fs, lr=lr, betas=betas,
                                      weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                                      master=master, schedule=schedule, warmup_steps=warmup_steps,
                                      total_steps=total_steps, seed=seed)
        elif self.ctx.world > 1:
            from ..parallel.zero import ShardedAdamW
            self.opt = ShardedAdamW(self.w, self.eng, self.ctx, lr=lr, betas=betas,
                                    weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                                    master=master, schedule=schedule, warmup_steps=warmup_steps,
                                    total_steps=total_steps, seed=seed, comm=comm)
        if self.w.ep is not None:
            from .optimizer import ListAdamW
            self.opt.local = ListAdamW(dict(self.w.expert_bufs), dict(self.eng.expert_grads), lr=lr, betas=betas,
                                       weight_decay=weight_decay, master=master, schedule=schedule,
                                       warmup_steps=warmup_steps, total_steps=total_steps, seed=seed)
        if self.ctx.world <= 1:
            self.opt = AdamW(self.w, self.eng, lr=lr, betas=betas, weight_decay=weight_decay,
                             max_grad_norm=max_grad_norm, master=master, schedule=schedule,
                             warmup_steps=warmup_steps, total_steps=total_steps, seed=seed)
        self._count = torch.zeros(1, dtype=torch.float32, device=dev)
        if recompute not in ("auto", "full", "none"):
            raise ValueError("recompute must be auto|full|none")
        self.recompute = recompute
        self.moment_offload = moment_offload
        self.reserve_bytes = int(activation_reserve_gb * 1e9)
        self._planned_tokens = None

    def _moment_shuttle(self, n_micro: int, micro_tokens: int):
        """On one GPU where the weights, gradients and fp32 moments leave no
        room to keep layer contexts, move the second moments to pinned host
        memory for the middle of the step (see :class:`MomentShuttle`)."""
        if self.moment_offload == "never" or self.ctx.world > 1 or self.ctx.device.type != "cuda":
            return None
        if not isinstance(self.opt, AdamW) or self.recompute != "auto" or self.cfg.is_moe or n_micro < 3:
            return None
        L = self.cfg.num_hidden_layers
        if self.moment_offload == "auto" and self.eng.keep_layers >= L:
            return None
        if getattr(self, "_shuttle", None) is None:
            self._shuttle = MomentShuttle(self, micro_tokens)
        self._shuttle.start(n_micro)
        return self._shuttle

    def plan_activations(self, micro_tokens: int) -> int:
        """Choose how many decoder layers keep their whole forward context
        (no recompute in the backward) for micro-batches of ``micro_tokens``.

        ``full``: none (every layer recomputes its GEMMs from its checkpointed
        input); ``none``: all; ``auto``: as many as fit in the HBM left after
        weights, gradients and optimizer state, minus a reserve for the head
        chunks and one recomputed layer. The choice is agreed as the minimum
        over ranks so every rank runs the same schedule."""
        L = self.cfg.num_hidden_layers
        if self.recompute == "full" or self.cfg.is_moe:
            keep = 0
        elif self.recompute == "none":
            keep = L
        elif self.ctx.device.type != "cuda":
            keep = 0
        else:
            free, _ = torch.cuda.mem_get_info(self.ctx.device)
            free += torch.cuda.memory_reserved(self.ctx.device) - torch.cuda.memory_allocated(self.ctx.device)
            per = self.eng.activation_bytes_per_layer(micro_tokens)
            budget = free - self.reserve_bytes - per
            keep = int(max(0, min(L, budget // per)))
        if self.ctx.world > 1:
            t = torch.tensor([float(keep)], device=self.ctx.device)
            self.ctx.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            keep = int(t.item())
        self.eng.keep_layers = keep
        self._planned_tokens = micro_tokens
        return keep

    @torch.no_grad()
    def train_step_device(self, ids: torch.Tensor, loss_mask: Optional[torch.Tensor] = None
                          ) -> torch.Tensor:
        """ids/loss_mask: [B, S] on the device. Returns the global mean loss (device)."""
        B, S = ids.shape
        if self._planned_tokens != min(self.mbs, B) * S:
            self.plan_activations(min(self.mbs, B) * S)
        lab = torch.zeros_like(ids, dtype=torch.bool)
        lab[:, :-1] = True if loss_mask is None else loss_mask[:, 1:].bool()
        self._count.fill_(0)
        self._count += lab.sum()
        self.ctx.all_reduce(self._count)
        self.eng.zero_grad()
        loss = torch.zeros((), dtype=torch.float32, device=ids.device)
        starts = list(range(0, B, self.mbs))
        shuttle = self._moment_shuttle(len(starts), min(self.mbs, B) * S)
        for i, s in enumerate(starts):
            if shuttle is not None:
                shuttle.before(i)
            b = Batch.from_dense(ids[s:s + self.mbs], None if loss_mask is None
                                 else loss_mask[s:s + self.mbs])
            coef = torch.where(b.targets >= 0, -1.0 / self._count, torch.zeros((), device=ids.device))
            out = self.eng.forward_backward(b, coef=coef)
            loss += out["loss"]
        if shuttle is not None:
            shuttle.finish()
        self.opt.step()
        self.ctx.all_reduce(loss)
        return loss

    @torch.no_grad()
    def train_step_sequences(self, seqs, label_masks, *, micro_tokens: int = 16384,
                             sample_weights=None) -> float:
        """Variable-length sequences (lists of token ids) packed into micro-batches
        of <= ``micro_tokens`` tokens; loss = global token mean of -logp over
        label tokens (optionally weighted per sample). Returns the loss."""
        dev = self.ctx.device
        n_lab = sum(int(torch.as_tensor(m)[1:].sum()) * (sample_weights[i] if sample_weights else 1.0)
                    for i, m in enumerate(label_masks))
        tot = torch.tensor([float(n_lab)], dtype=torch.float32, device=dev)
        self.ctx.all_reduce(tot)
        self.eng.zero_grad()
        loss = torch.zeros((), dtype=torch.float32, device=dev)
        order = list(range(len(seqs)))
        i = 0
        while i < len(order):
            chunk, ntok = [], 0
            while i < len(order) and (not chunk or ntok + len(seqs[order[i]]) <= micro_tokens):
                chunk.append(order[i])
                ntok += len(seqs[order[i]])
                i += 1
            b = Batch.from_sequences([torch.as_tensor(seqs[j]) for j in chunk],
                                     [torch.as_tensor(label_masks[j]) for j in chunk], device=dev)
            coef = torch.zeros(b.num_tokens, dtype=torch.float32)
            off = 0
            for j in chunk:
                L = len(seqs[j])
                w = sample_weights[j] if sample_weights else 1.0
                coef[off:off + L] = -w
                off += L
            coef = coef.to(dev) / tot
            coef = torch.where(b.targets >= 0, coef, torch.zeros_like(coef))
            loss += self.eng.forward_backward(b, coef=coef)["loss"]
        self.opt.step()
        self.ctx.all_reduce(loss)
        return float(loss.item())

    @torch.no_grad()
    def full_weights(self) -> Qwen3Weights:
        """The model with every unit materialised (gathers ZeRO-3 shards; for saving)."""
        if getattr(self, "fs", None) is None:
            return self.w
        full = Qwen3Weights(self.cfg, device=self.w.device, dtype=self.w.dtype, allocate=False,
                            pad_multiple=self.w.pad_multiple, ep=self.w.ep)
        full.bufs = [self.fs.full_unit(u).clone() if u in self.fs.pshard else self.w.bufs[u]
                     for u in range(self.w.num_units)]
        full.expert_bufs = self.w.expert_bufs
        return full

    @torch.no_grad()
    def load_checkpoint(self, path: str) -> None:
        """Load HF weights (re-sharding ZeRO-3 layer units)."""
        from ..models.hf_io import load_weights
        if getattr(self, "fs", None) is None:
            load_weights(self.w, path)
            return
        full = Qwen3Weights(self.cfg, device=self.w.device, dtype=self.w.dtype, init=False,
                            pad_multiple=self.w.pad_multiple, ep=self.w.ep)
        load_weights(full, path)
        r, s = self.ctx.rank, self.fs.s
        for u in range(self.w.num_units):
            if u in self.fs.pshard:
                self.fs.pshard[u].copy_(full.bufs[u][r * s:(r + 1) * s])
                if u in self.opt.master:
                    self.opt.master[u].copy_(self.fs.pshard[u].float())
            else:
                self.w.bufs[u].copy_(full.bufs[u])
        for u, b in full.expert_bufs.items():
            self.w.expert_bufs[u].copy_(b)
        self.fs.owner = [-1, -1]

    def train_step(self, ids_host: torch.Tensor, loss_mask_host: Optional[torch.Tensor] = None
                   ) -> float:
        """Host inputs in, host loss out (the end-to-end call)."""
        dev = self.ctx.device
        ids = ids_host.to(dev, non_blocking=True)
        mask = loss_mask_host.to(dev, non_blocking=True) if loss_mask_host is not None else None
        loss = float(self.train_step_device(ids, mask).item())
        if hasattr(self.eng.ep, "check_overflow"):
            self.eng.ep.check_overflow()          # one flag read per step (the step synchronised already)
        return loss


class MomentShuttle:
    """Second moments out of HBM for the middle micro-batches of a step.

    A 14B model on one GPU holds bf16 weights and gradients and fp32 moments
    (177 GB), so every layer recomputes its forward GEMMs in the backward. The
    shuttle copies the second moments (59 GB) to pinned host memory on a side
    stream while the first micro-batch runs, lets the middle micro-batches keep
    their whole layer contexts in the freed HBM (no recompute), and copies the
    moments back on the side stream while the last micro-batch runs with
    recompute, so neither copy is on the critical path. The optimizer step
    waits for the copy back."""

    def __init__(self, trainer: "CausalLMTrainer", micro_tokens: int):
        self.tr = trainer
        self.stream = torch.cuda.Stream(device=trainer.ctx.device)
        self.keys = sorted(trainer.opt.v)
        self.host = {}
        self.micro_tokens = micro_tokens
        self.ev = None
        self.n = 0
        self.keep_mid = None
        for k in self.keys:
            t = trainer.opt.v[k]
            try:
                self.host[k] = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            except RuntimeError:             # page-locking refused: pageable copies still work
                self.host[k] = torch.empty(t.shape, dtype=t.dtype)

    def start(self, n_micro: int) -> None:
        self.n = n_micro
        opt = self.tr.opt
        main = torch.cuda.current_stream()
        self.stream.wait_stream(main)                    # v is final after the previous step
        with torch.cuda.stream(self.stream):
            for k in self.keys:
                t = opt.v[k]
                self.host[k].copy_(t, non_blocking=True)
                t.record_stream(self.stream)
                opt.v[k] = None
            self.ev = torch.cuda.Event()
            self.ev.record()
        self.tr.eng.keep_layers = 0

    def before(self, i: int) -> None:
        eng = self.tr.eng
        if i == 1:
            self.ev.synchronize()                        # the moments have left HBM
            if self.keep_mid is None:
                torch.cuda.empty_cache()
                self.tr.plan_activations(self.micro_tokens)
                self.keep_mid = eng.keep_layers
            eng.keep_layers = self.keep_mid
        elif i == self.n - 1:
            eng.keep_layers = 0                          # room for the moments coming back
            main = torch.cuda.current_stream()
            opt = self.tr.opt
            for k in self.keys:
                opt.v[k] = torch.empty(self.host[k].shape, dtype=self.host[k].dtype, device=self.tr.ctx.device)
            self.stream.wait_stream(main)
            with torch.cuda.stream(self.stream):
                for k in self.keys:
                    opt.v[k].copy_(self.host[k], non_blocking=True)
                self.ev = torch.cuda.Event()
                self.ev.record()

    def finish(self) -> None:
        torch.cuda.current_stream().wait_event(self.ev)
