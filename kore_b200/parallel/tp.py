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
nothing crosses NVLink, and the shard tensors are refilled in place. All
ranks prefill their prompts together, then decode in lockstep; after each
step the finished sequences leave the batch (the active ones are compacted and
padded to a common multiple of 64 rows), and decoding ends when every rank's
sequences are done.
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
        """Weight sync after an optimizer step, in place and allocation-free:
        each shard tensor is refilled from strided views of the full layer
        (every rank holds the full updated parameters after its ZeRO step)."""
        c, r, D = self.cfg, self.rank, self.cfg.head_dim
        qd, kd, F = c.q_dim, c.kv_dim, c.intermediate_size
        nq, nk = self.hq * D, self.hkv * D
        for li, u in enumerate(range(1, weights.num_units - 1)):
            W, L = weights.views(u), self.layers[li]
            for k in ("ln1", "ln2", "q_norm", "k_norm"):
                if L[k].data_ptr() != W[k].data_ptr():
                    L[k].copy_(W[k])
            L["qkv"][:nq].copy_(W["qkv"][r * nq:(r + 1) * nq])
            L["qkv"][nq:nq + nk].copy_(W["qkv"][qd + r * nk: qd + (r + 1) * nk])
            L["qkv"][nq + nk:].copy_(W["qkv"][qd + kd + r * nk: qd + kd + (r + 1) * nk])
            L["o"].copy_(W["o"][:, r * nq:(r + 1) * nq])
            L["gate_up"][:self.F].copy_(W["gate_up"][r * self.F:(r + 1) * self.F])
            L["gate_up"][self.F:].copy_(W["gate_up"][F + r * self.F: F + (r + 1) * self.F])
            L["down"].copy_(W["down"][:, r * self.F:(r + 1) * self.F])
        for name, src in (("embed", weights.views(0)["embed"]),
                          ("norm", weights.views(weights.num_units - 1)["norm"]),
                          ("lm_head", weights.lm_head_weight())):
            dst = getattr(self, name)
            if dst.data_ptr() != src.data_ptr():
                dst.copy_(src)


class TPRolloutEngine:
    """``max_rows``: rows per rank in one forward chunk (prefill / extend are
    chunked to it; the GEMMs see ``world * max_rows`` rows). ``max_seqs``:
    sequences per rank. The KV cache (this rank's kv heads of every rank's
    sequences) is allocated on first use and can be released between
    rollouts (``release_cache``)."""

    def __init__(self, weights, ctx, *, max_rows: int = 4096, max_seqs: int = 64, max_seq_len: int = 8192,
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
        self.max_seq_len = max_seq_len
        self.max_pages = (max_seq_len + page_size - 1) // page_size
        self.n_pages = self.W * self.S * self.max_pages + 1
        self.dtype, self.dev = weights.dtype, weights.device
        self.kc: Optional[List[torch.Tensor]] = None
        self.vc: Optional[List[torch.Tensor]] = None
        self.pad_slot = (self.n_pages - 1) * page_size  # writes of padding rows land here
        self.cos, self.sin = ref.rope_tables(c.max_position_embeddings, self.D, c.rope_theta, self.dev)
        self._step = 0
        self.lens = [[0] * self.S for _ in range(self.W)]   # cached tokens of every rank's sequences

    # ------------------------------------------------------------ cache
    def kv_bytes(self) -> int:
        return 2 * self.cfg.num_hidden_layers * self.n_pages * self.ps * self.shard.hkv * self.D * \
            torch.empty((), dtype=self.dtype).element_size()

    def ensure_cache(self) -> None:
        if self.kc is None:
            shape = (self.n_pages * self.ps, self.shard.hkv, self.D)
            self.kc = [torch.empty(shape, dtype=self.dtype, device=self.dev) for _ in range(self.cfg.num_hidden_layers)]
            self.vc = [torch.empty(shape, dtype=self.dtype, device=self.dev) for _ in range(self.cfg.num_hidden_layers)]

    def release_cache(self) -> None:
        self.kc = self.vc = None
        self.lens = [[0] * self.S for _ in range(self.W)]
        if self.dev.type == "cuda":
            torch.cuda.empty_cache()

    def reset(self) -> None:
        """Forget every sequence (their pages are reused from position 0)."""
        self.lens = [[0] * self.S for _ in range(self.W)]

    def _page0(self, rank: int, i: int) -> int:
        return (rank * self.S + i) * self.max_pages

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

    # ------------------------------------------------------------ extend / generate
    def _extend(self, pending: Sequence[Sequence[int]]):
        """Feed every sequence's pending tokens into the cache (all ranks call
        together). Chunks of at most ``max_rows`` rows per rank; a chunk whose
        segments are all fresh whole sequences runs the flash-attention
        prefill, any other the paged kernel over the cache. Returns the
        last-token logits of my sequences that had pending tokens, and their ids."""
        W, ps, Rc = self.W, self.ps, self.R
        chunks: List[list] = []
        cur, used = [], 0
        for i, toks in enumerate(pending):
            off = 0
            while off < len(toks):
                take = min(len(toks) - off, Rc - used)
                cur.append((i, off, take, len(toks)))
                used += take
                off += take
                if used == Rc:
                    chunks.append(cur)
                    cur, used = [], 0
        if cur:
            chunks.append(cur)
        all_chunks = self.ctx.all_gather_object(chunks) if W > 1 else [chunks]
        nch = max(len(c) for c in all_chunks)
        scale = 1.0 / math.sqrt(self.D)
        C = ops.native()
        out = []
        for ci in range(nch):
            segs = [all_chunks[rk][ci] if ci < len(all_chunks[rk]) else [] for rk in range(W)]
            rows = max(64, (max(sum(t for _, _, t, _ in sg) for sg in segs) + 63) // 64 * 64)
            fresh = all(self.lens[rk][i] == 0 and off == 0 and take == tot
                        for rk in range(W) for i, off, take, tot in segs[rk])
            pos, slots, qs, lens_q, bt_rows = [], [], [0], [], []
            for rk in range(W):
                n_used = 0
                for i, off, take, tot in segs[rk]:
                    L0 = self.lens[rk][i]
                    assert L0 + take <= self.max_seq_len, "sequence exceeds max_seq_len"
                    pg = self._page0(rk, i)
                    for j in range(take):
                        pos.append(L0 + j)
                        slots.append((pg + (L0 + j) // ps) * ps + (L0 + j) % ps)
                    qs.append(qs[-1] + take)
                    lens_q.append(L0 + take)
                    bt_rows.append(pg)
                    n_used += take
                for _ in range(rows - n_used):       # padding rows: one-row segments on the pad slot
                    pos.append(0)
                    slots.append(self.pad_slot)
                    qs.append(qs[-1] + 1)
                    lens_q.append(1)
                    bt_rows.append(self.n_pages - 1)
            toks = torch.zeros(rows, dtype=torch.long)
            k = 0
            for i, off, take, tot in segs[self.r]:
                toks[k:k + take] = torch.tensor(list(pending[i][off:off + take]), dtype=torch.long)
                k += take
            x = ops.embed_fwd(toks.to(self.dev), self.shard.embed)
            pos_t = torch.tensor(pos, dtype=torch.int32, device=self.dev)
            slots_t = torch.tensor(slots, dtype=torch.int32, device=self.dev)
            qs_t = torch.tensor(qs, dtype=torch.int32, device=self.dev)
            max_q = max(b - a for a, b in zip(qs[:-1], qs[1:]))
            if fresh:
                def attn_fn(q, k_, v, li):
                    return attn.attn_fwd(q, k_, v, qs_t, max_q, scale)[0]
            else:
                lens_t = torch.tensor(lens_q, dtype=torch.int32, device=self.dev)
                bt = (torch.tensor(bt_rows, dtype=torch.int32)[:, None]
                      + torch.arange(self.max_pages, dtype=torch.int32)[None, :])
                bt = bt.clamp_(max=self.n_pages - 1).to(self.dev)

                def attn_fn(q, k_, v, li):
                    o = torch.empty_like(q)
                    C.paged_attention(q, self.kc[li], self.vc[li], bt, lens_t, qs_t, max_q, ps, scale, 1,
                                      o, None, None)
                    return o
            h = self._layers(x, rows, pos_t, slots_t, attn_fn)
            k, rows_i, ids_i = 0, [], []
            for i, off, take, tot in segs[self.r]:
                k += take
                if off + take == tot:                # this chunk ends sequence i's pending tokens
                    rows_i.append(k - 1)
                    ids_i.append(i)
            for rk in range(W):
                for i, off, take, tot in segs[rk]:
                    self.lens[rk][i] += take
            if rows_i:
                idx = torch.tensor(rows_i, dtype=torch.long, device=self.dev)
                out.append((self._logits(h.index_select(0, idx)), ids_i))
        return out

    @torch.no_grad()
    def generate(self, pending: Sequence[Sequence[int]], max_new: int, *, temperature: float = 1.0,
                 top_p: float = 1.0, eos_ids: Sequence[int] = (), seed: int = 0):
        """Extend my sequences by ``pending[i]`` (a fresh sequence's whole
        prompt, or the tokens since its last turn) and sample up to
        ``max_new`` tokens for each; every rank calls together. The last
        sampled token of a sequence is not fed: it heads its next ``pending``.
        Sequences with nothing pending are not generated. Returns per-sequence
        (tokens, log-probs)."""
        import torch.distributed as dist
        assert len(pending) <= self.S, "too many sequences for this engine"
        self.ensure_cache()
        C = ops.native()
        W, ps, S = self.W, self.ps, self.S
        n = len(pending)
        parts = self._extend(pending)
        out_tok: List[List[int]] = [[] for _ in range(n)]
        out_lp: List[List[float]] = [[] for _ in range(n)]
        done = [True] * S
        eos = set(int(e) for e in eos_ids)
        act: List[int] = []
        toks_l: List[int] = []
        lps_l: List[float] = []
        for lg, ids in parts:
            t, l = self._sample(lg, temperature, top_p, seed, len(ids))
            act += ids
            toks_l += t
            lps_l += l
        cur = (toks_l, lps_l) if act else None
        for i in act:
            done[i] = False
        scale = 1.0 / math.sqrt(self.D)
        done_dev = torch.zeros(S, dtype=torch.int32, device=self.dev)
        done_all = torch.empty(W * S, dtype=torch.int32, device=self.dev)
        step = 0
        while True:
            if cur is not None:
                tk, lp = cur
                for j, i in enumerate(act):
                    out_tok[i].append(int(tk[j]))
                    out_lp[i].append(float(lp[j]))
                    if int(tk[j]) in eos or len(out_tok[i]) >= max_new:
                        done[i] = True
            step += 1
            done_dev.copy_(torch.tensor([int(d) for d in done], dtype=torch.int32))
            if W > 1:
                dist.all_gather_into_tensor(done_all, done_dev, group=self.ctx.group)
            else:
                done_all.copy_(done_dev)
            allf = done_all.view(W, S).tolist()
            acts = [[i for i in range(S) if not allf[rk][i]] for rk in range(W)]
            if all(not a for a in acts) or step >= max_new:
                break
            # decode: only unfinished sequences are rows, compacted and padded
            # to a common multiple of 64 rows on every rank
            act = acts[self.r]
            rows_d = max(64, (max(len(a) for a in acts) + 63) // 64 * 64)
            pos_l, slot_l, lens_l, bt_rows = [], [], [], []
            for rk in range(W):
                for j in range(rows_d):
                    if j < len(acts[rk]):
                        i = acts[rk][j]
                        L = self.lens[rk][i]
                        assert L < self.max_seq_len, "sequence exceeds max_seq_len"
                        pg = self._page0(rk, i)
                        pos_l.append(L)
                        slot_l.append((pg + L // ps) * ps + L % ps)
                        lens_l.append(L + 1)
                        bt_rows.append(pg)
                    else:
                        pos_l.append(0)
                        slot_l.append(self.pad_slot)
                        lens_l.append(1)
                        bt_rows.append(self.n_pages - 1)
            for rk in range(W):
                for i in acts[rk]:
                    self.lens[rk][i] += 1
            feed = torch.zeros(rows_d, dtype=torch.long)
            if act:
                feed[:len(act)] = torch.tensor([out_tok[i][-1] for i in act], dtype=torch.long)
            pos_t = torch.tensor(pos_l, dtype=torch.int32, device=self.dev)
            slots_t = torch.tensor(slot_l, dtype=torch.int32, device=self.dev)
            lens_t = torch.tensor(lens_l, dtype=torch.int32, device=self.dev)
            bt_d = (torch.tensor(bt_rows, dtype=torch.int32)[:, None]
                    + torch.arange(self.max_pages, dtype=torch.int32)[None, :]).clamp_(max=self.n_pages - 1)
            bt_d = bt_d.to(self.dev)
            qs_t = torch.arange(W * rows_d + 1, dtype=torch.int32, device=self.dev)
            x = ops.embed_fwd(feed.to(self.dev), self.shard.embed)

            def dec_attn(q, k, v, li, bt_d=bt_d, lens_t=lens_t, qs_t=qs_t):
                o = torch.empty_like(q)
                C.paged_attention(q, self.kc[li], self.vc[li], bt_d, lens_t, qs_t, 1, ps, scale, 1, o, None, None)
                return o

            h = self._layers(x, rows_d, pos_t, slots_t, dec_attn)
            cur = self._sample(self._logits(h[:len(act)]) if act else None, temperature, top_p, seed, len(act))
        return out_tok, out_lp

    @torch.no_grad()
    def generate_static(self, prompts: Sequence[Sequence[int]], max_new: int, **kw):
        """One fresh generation per prompt (the cache is reset first)."""
        self.reset()
        return self.generate(prompts, max_new, **kw)

    def _sample(self, logits, temperature, top_p, seed, n):
        self._step += 1
        if logits is None or n == 0:
            return None
        tok = torch.empty(n, dtype=torch.long, device=self.dev)
        lp = torch.empty(n, dtype=torch.float32, device=self.dev)
        ops.native().sample_tokens(logits, float(temperature), float(top_p),
                                   (int(seed) * 1000003 + self.r) & 0x7FFFFFFF, self._step, tok, lp)
        return tok.tolist(), lp.tolist()
