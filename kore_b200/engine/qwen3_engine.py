"""Explicit forward/backward engine for Qwen3 dense causal LMs.

Instead of autograd over nn.Modules, one micro-batch of packed tokens goes
through hand-sequenced native kernels:

  forward  : embed -> L x [RMSNorm -> QKV GEMM -> q/k-norm+RoPE -> attention
             -> O GEMM (+residual, fused in the epilogue) -> RMSNorm ->
             gate|up GEMM -> SwiGLU -> down GEMM (+residual)] -> RMSNorm
  head     : lm_head in token chunks -> fused log-softmax/entropy/grad kernel
             (the [T, V] fp32 logits tensor never exists)
  backward : per layer, recompute the layer from its saved input (activation
             checkpointing: only L x [T, H] bf16 is kept), then dgrad/wgrad
             GEMMs that read transposed operands in place and accumulate weight
             gradients straight into the flat gradient buffer.

Losses are expressed through per-token coefficients c_t = dL/dlogp_t:
SFT/midtrain pass them up front (one pass); GRPO/DPO pass a callable that
maps the micro-batch's token log-probs to coefficients (two-phase head).

Reference parity: the step the reference runs inside HF Trainer / TRL
(kore/policy/sft.py:346-399, kore/policy/dpo.py:237-364) and its per-sample
GRPO backward (kore/policy/grpo.py:613-701).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Optional

import torch

from .. import ops
from ..models.qwen3 import Qwen3Weights
from ..ops import attention as attn
from ..ops import reference as ref


@dataclass
class Batch:
    """One packed micro-batch. ``targets`` = next token (or -1 = no loss)."""
    ids: torch.Tensor           # [T] int64
    targets: torch.Tensor       # [T] int64
    pos: torch.Tensor           # [T] int32 positions within each sequence
    cu_seqlens: torch.Tensor    # [n+1] int32
    max_seqlen: int

    @staticmethod
    def from_sequences(seqs: List[torch.Tensor], loss_masks: Optional[List[torch.Tensor]] = None,
                       device=None) -> "Batch":
        """Pack token sequences; target of position i is token i+1 of the same
        sequence (last position and masked positions get -1)."""
        ids, tg, pos, cu = [], [], [], [0]
        for i, s in enumerate(seqs):
            s = s.reshape(-1).long()
            n = s.numel()
            t = torch.full((n,), -1, dtype=torch.long)
            t[:-1] = s[1:]
            if loss_masks is not None:
                m = loss_masks[i].reshape(-1).bool()
                # loss_mask[j] marks token j as a label: it is predicted at j-1
                lab = torch.zeros(n, dtype=torch.bool)
                lab[:-1] = m[1:]
                t[~lab] = -1
            ids.append(s)
            tg.append(t)
            pos.append(torch.arange(n, dtype=torch.int32))
            cu.append(cu[-1] + n)
        dev = device or (seqs[0].device if seqs else "cpu")
        return Batch(torch.cat(ids).to(dev), torch.cat(tg).to(dev), torch.cat(pos).to(dev),
                     torch.tensor(cu, dtype=torch.int32, device=dev),
                     max(int(c1 - c0) for c0, c1 in zip(cu[:-1], cu[1:])))

    @staticmethod
    def from_dense(ids: torch.Tensor, loss_mask: Optional[torch.Tensor] = None) -> "Batch":
        """Pack a [B, S] block of equal-length sequences without host syncs.
        ``loss_mask[b, j]`` marks token j as a label (predicted from j-1)."""
        B, S = ids.shape
        dev = ids.device
        ids = ids.long()
        tg = torch.full_like(ids, -1)
        tg[:, :-1] = ids[:, 1:]
        if loss_mask is not None:
            lab = torch.zeros_like(loss_mask, dtype=torch.bool)
            lab[:, :-1] = loss_mask[:, 1:].bool()
            tg = torch.where(lab, tg, torch.full_like(tg, -1))
        pos = torch.arange(S, dtype=torch.int32, device=dev).repeat(B)
        cu = torch.arange(0, (B + 1) * S, S, dtype=torch.int32, device=dev)
        return Batch(ids.reshape(-1), tg.reshape(-1), pos, cu, S)

    @property
    def num_tokens(self) -> int:
        return int(self.ids.numel())


class Qwen3Engine:
    """Training/scoring engine over a :class:`Qwen3Weights`.

    ``grads`` are flat buffers matching the weight units (bf16 by default,
    fp32 optional); weight-gradient GEMMs accumulate into them across
    micro-batches until :meth:`zero_grad`.
    """

    def __init__(self, weights: Qwen3Weights, *, grad_dtype: Optional[torch.dtype] = None,
                 logits_chunk: int = 4096, temperature: float = 1.0, allocate_grads: bool = True,
                 save_attention: bool = True, grad_alloc=None):
        self.w = weights
        self.cfg = weights.cfg
        self.dev = weights.device
        self.dtype = weights.dtype
        self.grad_dtype = grad_dtype or self.dtype
        self.logits_chunk = logits_chunk
        # selective activation checkpointing: keep attention outputs (T x Hq*D
        # bf16 + lse per layer) so the backward recomputes only the GEMMs
        self.save_attention = save_attention
        # decoder layers (counted from the last one) whose whole forward context
        # is kept during forward_backward, so their backward recomputes nothing;
        # set by the trainer from the free HBM (0 = full activation checkpointing)
        self.keep_layers = 0
        self.ep = None          # expert-parallel dispatcher (kore_b200.parallel.ep) when attached
        self.param_hook = None  # full-sharding provider (kore_b200.parallel.fsdp.FullShard) when attached
        self.temperature = temperature
        c = self.cfg
        self.hq, self.hkv, self.D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        self.eps = c.rms_norm_eps
        self.cos, self.sin = ref.rope_tables(c.max_position_embeddings, c.head_dim, c.rope_theta,
                                             self.dev)
        self.grads: List[Optional[torch.Tensor]] = [None] * weights.num_units
        # expert-parallel runs: gradients of this rank's own experts (never reduced)
        self.expert_grads = {u: torch.zeros(b.numel(), dtype=self.grad_dtype, device=self.dev)
                             for u, b in weights.expert_bufs.items()} if allocate_grads else {}
        self._fresh = [True] * weights.num_units
        if allocate_grads:
            for u in range(weights.num_units):
                if grad_alloc is not None:
                    self.grads[u] = grad_alloc(weights.padded_numel(u), self.grad_dtype)
                    self.grads[u].zero_()
                else:
                    self.grads[u] = torch.zeros(weights.padded_numel(u), dtype=self.grad_dtype,
                                                device=self.dev)

    # ------------------------------------------------------------------ utils
    def zero_grad(self) -> None:
        """Mark gradients stale: the next backward overwrites instead of adding."""
        self._fresh = [True] * self.w.num_units
        if self.param_hook is not None:
            self.param_hook.zero_grad()
        for g in self.grads:
            if g is not None:
                g.zero_()
        for g in self.expert_grads.values():
            g.zero_()

    def grad_views(self, u: int):
        v = self.w.layouts[u].views(self.grads[u])
        if u in self.expert_grads:
            v.update(self.w.expert_layouts[u].views(self.expert_grads[u]))
        return v

    def _acc_vec(self, dst: torch.Tensor, src_f32: torch.Tensor) -> None:
        dst.add_(src_f32.to(dst.dtype))

    def _mm(self, a, b, **kw):
        kw.setdefault("out_dtype", self.dtype)
        return ops.mm(a, b, **kw)

    # ------------------------------------------------------------------ layer
    def _layer_fwd(self, u: int, x: torch.Tensor, b: Batch, keep: bool, attn_saved=None,
                   save_attn: Optional[list] = None):
        W = self.w.views(u)
        T = x.shape[0]
        qd, kd = self.hq * self.D, self.hkv * self.D
        f32 = dict(dtype=torch.float32, device=x.device)
        rstd1 = torch.empty(T, **f32)
        hn = ops.rmsnorm_fwd(x, W["ln1"], self.eps, rstd=rstd1)
        qkv = self._mm(hn, W["qkv"])
        qk = ops.qk_norm_rope_fwd(qkv, W["q_norm"], W["k_norm"], b.pos, self.cos, self.sin,
                                  self.hq, self.hkv, self.eps)
        q = qk[:, :qd].view(T, self.hq, self.D)
        k = qk[:, qd:].view(T, self.hkv, self.D)
        v = qkv[:, qd + kd:].view(T, self.hkv, self.D)
        if attn_saved is not None:
            o, lse = attn_saved           # selective checkpoint: no attention recompute
        else:
            o, lse = attn.attn_fwd(q, k, v, b.cu_seqlens, b.max_seqlen)
        if save_attn is not None:
            save_attn.append((o, lse))
        o2 = o.reshape(T, qd)
        x2 = self._mm(o2, W["o"], residual=x)
        rstd2 = torch.empty(T, **f32)
        hn2 = ops.rmsnorm_fwd(x2, W["ln2"], self.eps, rstd=rstd2)
        ctx = None
        if self.w.layouts[u].kind == "moe_layer":
            x3, mctx = self._moe_fwd(W, hn2, x2)
            if keep:
                ctx = dict(rstd1=rstd1, hn=hn, qkv=qkv, qk=qk, o=o, lse=lse, x2=x2, rstd2=rstd2, hn2=hn2)
                ctx.update(mctx)             # the expert-parallel context may carry its own hn2
            return x3, ctx
        gu = self._mm(hn2, W["gate_up"])
        a = ops.swiglu_fwd(gu)
        x3 = self._mm(a, W["down"], residual=x2)
        if keep:
            ctx = dict(rstd1=rstd1, hn=hn, qkv=qkv, qk=qk, o=o, lse=lse, x2=x2, rstd2=rstd2,
                       hn2=hn2, gu=gu, a=a)
        return x3, ctx

    # ------------------------------------------------------------------ MoE
    def _moe_fwd(self, W, hn2, x2):
        """Router -> top-k -> expert-major permutation -> grouped SwiGLU experts
        -> weighted combine (+ residual). Experts outside this rank's range (EP)
        are handled by the expert-parallel dispatcher when one is attached."""
        from ..ops import moe
        c = self.cfg
        logits = ops.mm(hn2, W["router"], out_dtype=torch.float32)
        probs, idx, wts = moe.route(logits, c.num_experts_per_tok, c.norm_topk_prob)
        if self.ep is not None:
            return self.ep.forward(self, W, hn2, x2, probs, idx, wts)
        # device routing plan (padded expert-major rows): no host synchronisation
        pl = moe.plan(idx, c.num_experts)
        xp = moe.plan_gather(hn2, pl)
        gu = moe.plan_mm(xp, W["experts_gate_up"], pl)
        a = ops.swiglu_fwd(gu)
        yp = moe.plan_mm(a, W["experts_down"], pl)
        x3 = moe.combine(yp, pl.pos, wts, resid=x2)
        return x3, dict(probs=probs, idx=idx, wts=wts, plan=pl, pos=pl.pos, xp=xp, gu=gu, a=a, yp=yp)

    def _moe_bwd(self, W, G, ctx, dx3, acc):
        """Returns d(hn2) of the MoE block; accumulates expert and router grads."""
        from ..ops import moe
        c = self.cfg
        if self.ep is not None:
            dhn2, dw = self.ep.backward(self, W, G, ctx, dx3)
        else:
            pl = ctx["plan"]
            dyp, dw = moe.combine_bwd(dx3, ctx["yp"], pl.pos, ctx["wts"])
            da = moe.plan_mm(dyp, W["experts_down"], pl, w_t=False)
            self._plan_wgrad(G["experts_down"], dyp, ctx["a"], pl)
            dgu = ops.swiglu_bwd(da, ctx["gu"], ctx["gu"])
            del da
            dxp = moe.plan_mm(dgu, W["experts_gate_up"], pl, w_t=False)
            self._plan_wgrad(G["experts_gate_up"], dgu, ctx["xp"], pl)
            dhn2 = moe.combine(dxp, pl.pos, None)
        dlogits = moe.route_bwd(ctx["probs"], ctx["idx"], ctx["wts"], dw, c.norm_topk_prob)
        dl = dlogits.to(self.dtype)
        self._mm(dl, W["router"], b_t=False, out=dhn2, accumulate=True)
        self._mm(dl, ctx["hn2"], a_t=True, b_t=False, out=G["router"], accumulate=acc)
        return dhn2

    def _plan_wgrad(self, Gw, dy, x, pl):
        """dW[e] += dy_e^T x_e for every expert in one launch when the gradient
        shapes tile (rows of dW a multiple of 128); else per expert."""
        from ..ops import moe
        if not dy.is_cuda or (Gw.shape[1] % 128 == 0 and Gw.shape[2] % 64 == 0):
            moe.plan_wgrad(dy, x, pl, Gw, accumulate=True)
        else:
            self._expert_wgrad(Gw, dy, x, pl.offsets.tolist())

    def _expert_wgrad(self, Gw, dy, x, offs, expert_base: int = 0):
        """dW[e] += dy_e^T x_e for each expert with rows (gradients are zeroed
        at zero_grad, so experts always accumulate)."""
        for e in range(len(offs) - 1):
            s, t = offs[e], offs[e + 1]
            if t > s:
                self._mm(dy[s:t], x[s:t], a_t=True, b_t=False, out=Gw[expert_base + e], accumulate=True)

    def _layer_bwd(self, u: int, x: torch.Tensor, dx3: torch.Tensor, ctx: dict, b: Batch):
        W = self.w.views(u)
        G = self.grad_views(u)
        acc = not self._fresh[u]
        T = x.shape[0]
        qd, kd = self.hq * self.D, self.hkv * self.D
        # MLP (dense SwiGLU or MoE experts)
        if self.w.layouts[u].kind == "moe_layer":
            dhn2 = self._moe_bwd(W, G, ctx, dx3, acc)
        else:
            da = self._mm(dx3, W["down"], b_t=False)                       # [T, F]
            self._mm(dx3, ctx["a"], a_t=True, b_t=False, out=G["down"], accumulate=acc)
            dgu = ops.swiglu_bwd(da, ctx["gu"], ctx["gu"])                  # in place
            del da
            dhn2 = self._mm(dgu, W["gate_up"], b_t=False)                  # [T, H]
            self._mm(dgu, ctx["hn2"], a_t=True, b_t=False, out=G["gate_up"], accumulate=acc)
            del dgu
        dw = torch.zeros(self.cfg.hidden_size, dtype=torch.float32, device=x.device)
        dx2 = ops.rmsnorm_bwd(dhn2, ctx["x2"], W["ln2"], ctx["rstd2"], dres=dx3, dw=dw)
        self._acc_norm(G["ln2"], dw, acc)
        del dhn2
        # attention
        do = self._mm(dx2, W["o"], b_t=False)                          # [T, qd]
        self._mm(dx2, ctx["o"].reshape(T, qd), a_t=True, b_t=False, out=G["o"], accumulate=acc)
        qk, qkv = ctx["qk"], ctx["qkv"]
        dqk = torch.empty_like(qk)
        dqkv = torch.empty_like(qkv)
        attn.attn_bwd(do.view(T, self.hq, self.D), qk[:, :qd].view(T, self.hq, self.D),
                      qk[:, qd:].view(T, self.hkv, self.D),
                      qkv[:, qd + kd:].view(T, self.hkv, self.D), ctx["o"], ctx["lse"],
                      b.cu_seqlens, b.max_seqlen,
                      dq=dqk[:, :qd].view(T, self.hq, self.D),
                      dk=dqk[:, qd:].view(T, self.hkv, self.D),
                      dv=dqkv[:, qd + kd:].view(T, self.hkv, self.D))
        del do
        dqw = torch.zeros(self.D, dtype=torch.float32, device=x.device)
        dkw = torch.zeros(self.D, dtype=torch.float32, device=x.device)
        ops.qk_norm_rope_bwd(dqk, qkv, W["q_norm"], W["k_norm"], b.pos, self.cos, self.sin,
                             dqkv, dqw, dkw, self.hq, self.hkv, self.eps)
        self._acc_norm(G["q_norm"], dqw, acc)
        self._acc_norm(G["k_norm"], dkw, acc)
        del dqk
        dhn = self._mm(dqkv, W["qkv"], b_t=False)
        self._mm(dqkv, ctx["hn"], a_t=True, b_t=False, out=G["qkv"], accumulate=acc)
        del dqkv
        dw.zero_()
        dx = ops.rmsnorm_bwd(dhn, x, W["ln1"], ctx["rstd1"], dres=dx2, dw=dw)
        self._acc_norm(G["ln1"], dw, acc)
        self._fresh[u] = False
        return dx

    def _acc_norm(self, g: torch.Tensor, dw32: torch.Tensor, acc: bool) -> None:
        if acc:
            g.add_(dw32.to(g.dtype))
        else:
            g.copy_(dw32.to(g.dtype))

    # ------------------------------------------------------------------ head
    def _head_logits(self, hn_rows: torch.Tensor) -> torch.Tensor:
        return self._mm(hn_rows, self.w.lm_head_weight())

    def _head_stats(self, hn: torch.Tensor, targets: torch.Tensor, rows: torch.Tensor,
                    want_entropy: bool):
        """log p(target) (and entropy) for the selected rows, chunked."""
        n = rows.numel()
        lp = torch.zeros(n, dtype=torch.float32, device=hn.device)
        ent = torch.zeros(n, dtype=torch.float32, device=hn.device) if want_entropy else None
        for s in range(0, n, self.logits_chunk):
            r = rows[s: s + self.logits_chunk]
            logits = self._head_logits(hn.index_select(0, r))
            a, e, _ = ops.logprob(logits, targets.index_select(0, r), self.temperature,
                                  want_entropy=want_entropy)
            lp[s: s + r.numel()] = a
            if want_entropy:
                ent[s: s + r.numel()] = e
            del logits
        return lp, ent

    def _head_bwd(self, hn: torch.Tensor, targets: torch.Tensor, rows: torch.Tensor,
                  coef: torch.Tensor) -> torch.Tensor:
        """dL/dhn for L = sum coef * logp over the selected rows; accumulates lm_head grads."""
        u_head = self.w.num_units - 1
        u_lm = 0 if self.cfg.tie_word_embeddings else u_head
        Glm = (self.grad_views(0)["embed"] if self.cfg.tie_word_embeddings
               else self.grad_views(u_head)["lm_head"])
        Wlm = self.w.lm_head_weight()
        dhn = torch.zeros_like(hn)
        self._last_rows_logp = torch.zeros(rows.numel(), dtype=torch.float32, device=hn.device)
        for s in range(0, rows.numel(), self.logits_chunk):
            r = rows[s: s + self.logits_chunk]
            hrows = hn.index_select(0, r)
            logits = self._head_logits(hrows)
            lp, _, _ = ops.logprob(logits, targets.index_select(0, r), self.temperature,
                                   coef=coef[s: s + r.numel()], write_grad=True)
            self._last_rows_logp[s: s + r.numel()] = lp
            dh = self._mm(logits, Wlm, b_t=False)
            dhn.index_copy_(0, r, dh)
            self._mm(logits, hrows, a_t=True, b_t=False, out=Glm, accumulate=not self._fresh[u_lm])
            self._fresh[u_lm] = False
            del logits, dh, hrows
        return dhn

    # ------------------------------------------------------------------ public
    def activation_bytes_per_layer(self, tokens: int) -> int:
        """HBM a dense layer's kept forward context takes for ``tokens`` tokens
        beyond what selective checkpointing keeps anyway (input, attention
        output and logsumexp)."""
        c = self.cfg
        qd, kd = self.hq * self.D, self.hkv * self.D
        H, F = c.hidden_size, c.intermediate_size
        elems = H + (qd + 2 * kd) + (qd + kd) + H + H + 2 * F + F   # hn qkv qk x2 hn2 gu a
        return tokens * (elems * self.w.dtype.itemsize + 8)           # + two fp32 rstd

    def _kept(self, u: int) -> bool:
        return self.keep_layers > 0 and u > self.w.num_units - 2 - self.keep_layers

    @torch.no_grad()
    def forward_hidden(self, b: Batch, checkpoints: Optional[list] = None,
                       attn_saves: Optional[list] = None, contexts: Optional[dict] = None) -> torch.Tensor:
        """Forward to the last hidden state. ``checkpoints`` collects each
        layer's input; ``attn_saves`` (selective checkpointing) also keeps each
        layer's attention output and logsumexp so the backward does not
        recompute attention; ``contexts`` receives the whole forward context of
        the layers selected by ``keep_layers`` (no recompute at all)."""
        x = ops.embed_fwd(b.ids, self.w.views(0)["embed"])
        hook = self.param_hook
        last = self.w.num_units - 2
        for u in range(1, self.w.num_units - 1):
            if checkpoints is not None:
                checkpoints.append(x)
            if hook is not None:
                hook.acquire(u, u + 1 if u < last else None)
            if contexts is not None and self._kept(u) and self.w.layouts[u].kind != "moe_layer":
                xin = x
                x, contexts[u] = self._layer_fwd(u, x, b, keep=True)
                if attn_saves is not None:
                    attn_saves.append(None)
                del xin
            else:
                x, _ = self._layer_fwd(u, x, b, keep=False, save_attn=attn_saves)
        return x

    @torch.no_grad()
    def token_logprobs_many(self, batches: List[Batch], want_entropy: bool = False):
        """``token_logprobs`` of several micro-batches, layer-major: each
        decoder layer is acquired once and applied to every batch's hidden
        states before the next layer. With a parameter provider that streams
        layers from host memory or gathers them over ranks, the weights then
        move once per call instead of once per micro-batch (the hidden states
        of all batches stay resident)."""
        xs = [ops.embed_fwd(b.ids, self.w.views(0)["embed"]) for b in batches]
        hook = self.param_hook
        last = self.w.num_units - 2
        for u in range(1, self.w.num_units - 1):
            if hook is not None:
                hook.acquire(u, u + 1 if u < last else None)
            for i, b in enumerate(batches):
                xs[i], _ = self._layer_fwd(u, xs[i], b, keep=False)
            if hook is not None and hasattr(hook, "release"):
                hook.release(u)
        return [self._logprobs_from_hidden(x, b, want_entropy) for x, b in zip(xs, batches)]

    @torch.no_grad()
    def token_logprobs(self, b: Batch, want_entropy: bool = False):
        """Per-token log p(target) (0 where target == -1), optional entropy."""
        return self._logprobs_from_hidden(self.forward_hidden(b), b, want_entropy)

    def _logprobs_from_hidden(self, x: torch.Tensor, b: Batch, want_entropy: bool):
        Wn = self.w.views(self.w.num_units - 1)["norm"]
        hn = ops.rmsnorm_fwd(x, Wn, self.eps)
        rows = torch.nonzero(b.targets >= 0).reshape(-1)
        lp_rows, ent_rows = self._head_stats(hn, b.targets, rows, want_entropy)
        lp = torch.zeros(b.num_tokens, dtype=torch.float32, device=x.device)
        lp[rows] = lp_rows
        ent = None
        if want_entropy:
            ent = torch.zeros(b.num_tokens, dtype=torch.float32, device=x.device)
            ent[rows] = ent_rows
        return lp, ent

    @torch.no_grad()
    def forward_backward(self, b: Batch, coef: Optional[torch.Tensor] = None,
                         coef_fn: Optional[Callable[[torch.Tensor], tuple]] = None) -> dict:
        """One micro-batch forward + backward.

        ``coef`` [T]: fixed dL/dlogp_t (0 for tokens without loss).
        ``coef_fn(logp[T]) -> (coef[T], loss_value)``: computed from this
        micro-batch's log-probs (two-phase head, for GRPO/DPO-style losses).
        Returns {"loss", "logp" (the rows' log-probs, [T])}.
        """
        assert (coef is None) != (coef_fn is None), "pass exactly one of coef / coef_fn"
        ckpts: list = []
        asaves: Optional[list] = [] if self.save_attention else None
        kept: dict = {}
        x = self.forward_hidden(b, ckpts, asaves, kept)
        uh = self.w.num_units - 1
        Wn = self.w.views(uh)["norm"]
        T = b.num_tokens
        rstd = torch.empty(T, dtype=torch.float32, device=x.device)
        hn = ops.rmsnorm_fwd(x, Wn, self.eps, rstd=rstd)
        valid = b.targets >= 0
        if coef is not None:
            valid = valid & (coef != 0)
        rows = torch.nonzero(valid).reshape(-1)
        lp_full = torch.zeros(T, dtype=torch.float32, device=x.device)
        if coef_fn is not None:
            lp_rows, _ = self._head_stats(hn, b.targets, rows, False)
            lp_full[rows] = lp_rows
            coef_full, loss = coef_fn(lp_full)
            coef_rows = coef_full.float()[rows]
        else:
            coef_rows = coef.float()[rows]
            loss = None
        dhn = self._head_bwd(hn, b.targets, rows, coef_rows)
        if coef_fn is None:
            # the gradient pass also produced log p(target) for the loss rows
            lp_full[rows] = self._last_rows_logp
            loss = (coef_rows * self._last_rows_logp).sum()
        dw = torch.zeros(self.cfg.hidden_size, dtype=torch.float32, device=x.device)
        dx = ops.rmsnorm_bwd(dhn, x, Wn, rstd, dw=dw)
        self._acc_norm(self.grad_views(uh)["norm"], dw, not self._fresh[uh])
        self._fresh[uh] = False
        del dhn, hn, x
        for u in range(self.w.num_units - 2, 0, -1):
            xin = ckpts[u - 1]
            saved = asaves[u - 1] if asaves is not None else None
            if self.param_hook is not None:
                self.param_hook.acquire(u, u - 1 if u > 1 else None)
                self.param_hook.begin_bwd(u)
            ctx = kept.pop(u, None)
            if ctx is None:
                _, ctx = self._layer_fwd(u, xin, b, keep=True, attn_saved=saved)
            dx = self._layer_bwd(u, xin, dx, ctx, b)
            if self.param_hook is not None:
                self.param_hook.end_bwd(u)
            del ctx, saved
            ckpts[u - 1] = None
            if asaves is not None:
                asaves[u - 1] = None
        # embedding
        Ge = self.grad_views(0)["embed"]
        if self._fresh[0] and not self.cfg.tie_word_embeddings:
            Ge.zero_()
        ops.embed_bwd(b.ids, dx, Ge)
        self._fresh[0] = False
        return {"loss": loss, "logp": lp_full}

    def sft_coef(self, b: Batch, normalizer: Optional[float] = None) -> torch.Tensor:
        """coef for mean token cross-entropy over the batch's labelled tokens
        (loss = -sum logp / normalizer)."""
        valid = (b.targets >= 0).float()
        n = normalizer if normalizer is not None else max(1.0, float(valid.sum()))
        return -valid / n
