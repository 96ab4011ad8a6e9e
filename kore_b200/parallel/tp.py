"""Tensor-parallel rollout engine over NVLink peer memory (path c + e).

Layout (sequence-parallel TP): every rank owns a block of sequences (its
rows) and 1/W of every layer's heads and FFN columns; embedding, final norm
and lm_head are replicated, so sampling and the residual stream stay local.
Per decoder layer:

  reduce(+residual)+RMSNorm of my rows -> heap       (fused kernel)
  QKV   = all-gather->GEMM: at kernel start the GEMM's CTAs copy each peer's
          64-row blocks of normed activations into a local staging buffer
          (every row crosses NVLink once) and flag them; a tile waits for its
          blocks and TMA-loads them locally, starting on this rank's own rows,
          so the copies overlap the first tiles. Computes my heads for ALL rows
  attention on my heads for all sequences (KV cache holds my kv heads only)
  O     = GEMM->reduce-scatter: the epilogue stores each output row into its
          owner's slot buffer with P2P stores; the owner sums the W slots in
          the next reduce+norm kernel
  gate|up (AG->GEMM), SwiGLU, down (GEMM->RS) likewise.

Weight sync (trainer -> rollout, path e): after a ZeRO step every rank holds
the full updated parameters, so each rank copies its own TP shard locally;
nothing crosses NVLink. Generation here is lockstep (static batch): all
ranks prefill their prompts, then decode ``max_new`` steps together; rows of
finished sequences keep decoding and are truncated at their stop token.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence

import torch

from .. import ops
from ..ops import attention as attn
from ..ops import reference as ref
from .symmetric import SymmetricHeap


class TPShard:
    """This rank's slice of every layer (heads / FFN columns)."""

    def __init__(self, weights, rank: int, world: int):
        c = weights.cfg
        self.cfg = c
        if c.num_attention_heads % world or c.num_key_value_heads % world or c.intermediate_size % world:
            raise ValueError("heads and FFN must be divisible by the TP size")
        self.rank, self.world = rank, world
        self.hq, self.hkv = c.num_attention_heads // world, c.num_key_value_heads // world
        self.F = c.intermediate_size // world
        self.layers: List[Dict[str, torch.Tensor]] = []
        D = c.head_dim
        for u in range(1, weights.num_units - 1):
            W = weights.views(u)
            qd, kd = c.q_dim, c.kv_dim
            q = W["qkv"][rank * self.hq * D:(rank + 1) * self.hq * D]
            k = W["qkv"][qd + rank * self.hkv * D: qd + (rank + 1) * self.hkv * D]
            v = W["qkv"][qd + kd + rank * self.hkv * D: qd + kd + (rank + 1) * self.hkv * D]
            F = c.intermediate_size
            g = W["gate_up"][rank * self.F:(rank + 1) * self.F]
            up = W["gate_up"][F + rank * self.F: F + (rank + 1) * self.F]
            self.layers.append({
                "ln1": W["ln1"], "ln2": W["ln2"], "q_norm": W["q_norm"], "k_norm": W["k_norm"],
                "qkv": torch.cat([q, k, v]).contiguous(),
                "o": W["o"][:, rank * self.hq * D:(rank + 1) * self.hq * D].contiguous(),
                "gate_up": torch.cat([g, up]).contiguous(),
                "down": W["down"][:, rank * self.F:(rank + 1) * self.F].contiguous()})
        self.embed = weights.views(0)["embed"]
        self.norm = weights.views(weights.num_units - 1)["norm"]
        self.lm_head = weights.lm_head_weight()

    @torch.no_grad()
    def sync_from(self, weights) -> None:
        """Weight sync after an optimizer step: local strided copies only."""
        fresh = TPShard(weights, self.rank, self.world)
        for a, b in zip(self.layers, fresh.layers):
            for k in a:
                if a[k].data_ptr() != b[k].data_ptr():
                    a[k].copy_(b[k])


class TPRolloutEngine:
    def __init__(self, weights, ctx, *, max_rows: int = 16384, max_seqs: int = 64, max_seq_len: int = 8192,
                 page_size: int = 64):
        c = weights.cfg
        self.cfg, self.ctx = c, ctx
        self.W, self.r = ctx.world, ctx.rank
        self.shard = TPShard(weights, self.r, self.W)
        self.D = c.head_dim
        self.eps = c.rms_norm_eps
        self.R = (max_rows + 63) // 64 * 64
        self.S = max_seqs
        self.ps = page_size
        H = c.hidden_size
        self.heap = SymmetricHeap(ctx, (self.R * H + self.W * self.R * max(H, 1)) * 2 + (1 << 20))
        self.o_hn, self.hn = self.heap.alloc(self.R * H)
        self.o_slots, self.slots = self.heap.alloc(self.W * self.R * H)
        C = ops.native()
        self.hn_peers = C.symm_peer_addrs(self.heap.id, self.o_hn)
        # all-gather staging: each peer row block is copied here once per GEMM
        self.stage = torch.empty(self.W * self.R * H, dtype=weights.dtype, device=weights.device)
        self.flags = torch.zeros(self.W * self.R // 64, dtype=torch.int32, device=weights.device)
        self.ag_epoch = 0
        self.slot_peers = C.symm_peer_addrs(self.heap.id, self.o_slots)
        self.max_pages = (max_seq_len + page_size - 1) // page_size
        n_pages = self.W * self.S * self.max_pages + 1
        dev = weights.device
        self.kc = [torch.empty(n_pages * page_size, self.shard.hkv, self.D, dtype=weights.dtype, device=dev)
                   for _ in range(c.num_hidden_layers)]
        self.vc = [torch.empty_like(t) for t in self.kc]
        self.pad_slot = (n_pages - 1) * page_size      # writes of padding rows land here
        self.cos, self.sin = ref.rope_tables(c.max_position_embeddings, self.D, c.rope_theta, dev)
        self.dev = dev
        self._step = 0

    # ------------------------------------------------------------ layer
    def _layers(self, x, rows: int, pos, slots, attn_fn):
        """x: [rows, H] my rows (residual stream); all ranks call with equal rows."""
        C = ops.native()
        c = self.cfg
        H = c.hidden_size
        W, r = self.W, self.r
        M = W * rows
        hq, hkv, D = self.shard.hq, self.shard.hkv, self.D
        hn = self.hn[: rows * H].view(rows, H)
        ops.rmsnorm_fwd(x, self.shard.layers[0]["ln1"], self.eps, out=hn)
        for li, L in enumerate(self.shard.layers):
            self.heap.barrier()                                    # every rank's normed rows ready
            qkv = torch.empty(M, (hq + 2 * hkv) * D, dtype=x.dtype, device=x.device)
            C.gemm_tp_bf16(None, self.hn_peers, H, M, L["qkv"], qkv, [], 0, rows, r, *self._ag())
            qk = ops.qk_norm_rope_fwd(qkv, L["q_norm"], L["k_norm"], pos, self.cos, self.sin, hq, hkv, self.eps)
            q = qk[:, : hq * D].view(M, hq, D)
            k = qk[:, hq * D:].view(M, hkv, D)
            v = qkv[:, (hq + hkv) * D:].view(M, hkv, D)
            C.kv_append(k, v, slots, self.kc[li], self.vc[li])
            o = attn_fn(q, k, v, li)
            self.heap.barrier()                                    # peers done reading my hn / slots free
            C.gemm_tp_bf16(o.reshape(M, hq * D), [], 0, M, L["o"], None, self.slot_peers, H, rows, r)
            self.heap.barrier()                                    # all partial rows delivered
            C.tp_reduce_norm(self.slots, W, rows, x, L["ln2"], hn, self.eps)
            self.heap.barrier()
            gu = torch.empty(M, 2 * self.shard.F, dtype=x.dtype, device=x.device)
            C.gemm_tp_bf16(None, self.hn_peers, H, M, L["gate_up"], gu, [], 0, rows, r, *self._ag())
            a = ops.swiglu_fwd(gu)
            self.heap.barrier()
            C.gemm_tp_bf16(a, [], 0, M, L["down"], None, self.slot_peers, H, rows, r)
            self.heap.barrier()
            nxt = self.shard.layers[li + 1]["ln1"] if li + 1 < len(self.shard.layers) else self.shard.norm
            C.tp_reduce_norm(self.slots, W, rows, x, nxt, hn, self.eps)
        return hn                                                  # final-normed rows

    def _ag(self):
        self.ag_epoch += 1
        return self.stage, self.flags, self.ag_epoch

    def _logits(self, h_rows):
        return ops.mm(h_rows, self.shard.lm_head)

    # ------------------------------------------------------------ generate
    @torch.no_grad()
    def generate_static(self, prompts: Sequence[Sequence[int]], max_new: int, *, temperature: float = 1.0,
                        top_p: float = 1.0, eos_ids: Sequence[int] = (), seed: int = 0):
        """Lockstep generation of this rank's prompts (all ranks must call)."""
        C = ops.native()
        n = len(prompts)
        assert n <= self.S, "too many sequences for this engine"
        lens = [len(p) for p in prompts]
        info = self.ctx.all_gather_object(lens)                    # every rank's prompt lengths
        W, ps, S = self.W, self.ps, self.S
        rows_p = max(64, (max(sum(l) for l in info) + 63) // 64 * 64)
        assert rows_p <= self.R, "prefill rows exceed the engine capacity"

        def page0(rank, i):
            return ((rank * S) + i) * self.max_pages

        # ---- prefill: my prompt tokens, padded to rows_p; block tables global and identical on all ranks
        toks = torch.zeros(rows_p, dtype=torch.long)
        cat = [t for p in prompts for t in p]
        toks[: len(cat)] = torch.tensor(cat, dtype=torch.long)
        x = ops.embed_fwd(toks.to(self.dev), self.shard.embed)
        pos_all, slot_all, cu = [], [], [0]
        for rk in range(W):
            used = 0
            for i, L in enumerate(info[rk]):
                pos_all += list(range(L))
                slot_all += [page0(rk, i) * ps + j for j in range(L)]
                cu.append(cu[-1] + L)
                used += L
            pad = rows_p - used
            if pad:
                pos_all += [0] * pad
                slot_all += [self.pad_slot] * pad
                cu.append(cu[-1] + pad)
        pos_t = torch.tensor(pos_all, dtype=torch.int32, device=self.dev)
        slots_t = torch.tensor(slot_all, dtype=torch.int32, device=self.dev)
        cu_t = torch.tensor(cu, dtype=torch.int32, device=self.dev)
        maxlen = max([rows_p] + [max(l) if l else 0 for l in info])
        scale = 1.0 / math.sqrt(self.D)
        h = self._layers(x, rows_p, pos_t, slots_t,
                         lambda q, k, v, li: attn.attn_fwd(q, k, v, cu_t, maxlen, scale)[0])
        last = torch.tensor([sum(lens[: i + 1]) - 1 for i in range(n)], dtype=torch.long, device=self.dev)
        out_tok = [[] for _ in range(n)]
        out_lp = [[] for _ in range(n)]
        done = [False] * n
        eos = set(int(e) for e in eos_ids)
        cur = self._sample(self._logits(h.index_select(0, last)) if n else None, temperature, top_p, seed, n)
        # ---- decode: rows = S per rank (padded to 64)
        rows_d = max(64, (S + 63) // 64 * 64)
        lengths = [list(l) + [0] * (S - len(l)) for l in info]
        bt = torch.zeros(W * rows_d, self.max_pages, dtype=torch.int32)
        for rk in range(W):
            for i in range(S):
                bt[rk * rows_d + i] = torch.arange(page0(rk, i), page0(rk, i) + self.max_pages, dtype=torch.int32)
        bt = bt.to(self.dev)
        for step in range(max_new):
            if cur is not None:
                tk, lp = cur
                for i in range(n):
                    if not done[i]:
                        out_tok[i].append(int(tk[i]))
                        out_lp[i].append(float(lp[i]))
                        if int(tk[i]) in eos or len(out_tok[i]) >= max_new:
                            done[i] = True
            if step == max_new - 1:
                break
            feed = torch.zeros(rows_d, dtype=torch.long)
            if n:
                feed[:n] = torch.tensor([t[-1] if t else 0 for t in out_tok], dtype=torch.long)
            pos_l, slot_l, lens_l = [], [], []
            for rk in range(W):
                for i in range(rows_d):
                    L = lengths[rk][i] + step if i < S and i < len(info[rk]) else 0
                    pos_l.append(L)
                    valid = i < len(info[rk])
                    slot_l.append(page0(rk, i) * ps + L if valid else self.pad_slot)
                    lens_l.append(L + 1 if valid else 1)
            pos_t = torch.tensor(pos_l, dtype=torch.int32, device=self.dev)
            slots_t = torch.tensor(slot_l, dtype=torch.int32, device=self.dev)
            lens_t = torch.tensor(lens_l, dtype=torch.int32, device=self.dev)
            qs_t = torch.arange(W * rows_d + 1, dtype=torch.int32, device=self.dev)
            x = ops.embed_fwd(feed.to(self.dev), self.shard.embed)

            def dec_attn(q, k, v, li):
                o = torch.empty_like(q)
                C.paged_attention(q, self.kc[li], self.vc[li], bt, lens_t, qs_t, 1, ps, scale, 1, o, None, None)
                return o

            h = self._layers(x, rows_d, pos_t, slots_t, dec_attn)
            cur = self._sample(self._logits(h[:n]) if n else None, temperature, top_p, seed, n)
        return out_tok, out_lp

    def _sample(self, logits, temperature, top_p, seed, n):
        self._step += 1
        if logits is None or n == 0:
            return None
        tok = torch.empty(n, dtype=torch.long, device=self.dev)
        lp = torch.empty(n, dtype=torch.float32, device=self.dev)
        ops.native().sample_tokens(logits, float(temperature), float(top_p),
                                   (int(seed) * 1000003 + self.r) & 0x7FFFFFFF, self._step, tok, lp)
        return tok.tolist(), lp.tolist()
