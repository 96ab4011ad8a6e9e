"""Rollout (generation) engine: paged KV cache + continuous batching.

* KV cache: per layer one K and one V pool of ``num_pages * page_size`` token
  slots ([slots, Hkv, 128] bf16). Sequences own page lists (block tables);
  pages return to a free list when a sequence finishes, and waiting prompts
  are admitted as soon as pages and batch slots free up (continuous
  batching). Sequences of one GRPO group can share their prompt's full pages
  (``share_prefix``): the prompt is prefilled once and the group's samples
  reference the same pages.
* Prefill of fresh prompts runs the packed varlen tcgen05 flash-attention
  kernel; later tokens (decode, and multi-turn "extend" chunks) run the
  paged split-KV attention kernel. Every GEMM is the tcgen05 GEMM.
* Sampling (temperature, top-p, Gumbel-max) and the sampled token's
  log-prob come from one fused kernel per step.

The engine reads weights from a :class:`Qwen3Weights` (on one GPU the
trainer's own buffers, so weight sync is free; with tensor parallelism the
trainer->rollout broadcast re-shards into the engine's layout).

Reference parity: replaces HF ``model.generate`` on a dense cache
(kore/policy/grpo.py:2365-2500, :2667-2698) and the eval-time vLLM wrapper
(kore/policy/serve.py:44-131).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from .. import ops
from ..models.qwen3 import Qwen3Weights
from ..ops import attention as attn
from ..ops import reference as ref


@dataclass
class GenRequest:
    prompt: List[int]
    max_new_tokens: int
    rid: int = 0
    share_key: Optional[object] = None  # requests with the same key share prompt pages


@dataclass
class GenResult:
    rid: int
    tokens: List[int]
    logps: List[float]
    finish_reason: str


@dataclass
class _Seq:
    req: GenRequest
    pages: List[int]
    shared_pages: int
    length: int                     # tokens whose K/V are in the cache
    pending: List[int]              # tokens to feed next step (not yet in cache)
    out: List[int] = field(default_factory=list)
    logps: List[float] = field(default_factory=list)
    done: bool = False
    reason: str = ""


class PagedKVCache:
    def __init__(self, num_layers: int, num_pages: int, page_size: int, hkv: int, head_dim: int,
                 device, dtype=torch.bfloat16):
        self.page_size = page_size
        self.num_pages = num_pages
        slots = num_pages * page_size
        self.k = [torch.empty(slots, hkv, head_dim, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v = [torch.empty(slots, hkv, head_dim, dtype=dtype, device=device) for _ in range(num_layers)]
        self.free: List[int] = list(range(num_pages - 1, -1, -1))
        self.refcount = [0] * num_pages

    def alloc(self, n: int) -> Optional[List[int]]:
        if n > len(self.free):
            return None
        out = [self.free.pop() for _ in range(n)]
        for p in out:
            self.refcount[p] = 1
        return out

    def retain(self, pages: Sequence[int]) -> None:
        for p in pages:
            self.refcount[p] += 1

    def release(self, pages: Sequence[int]) -> None:
        for p in pages:
            self.refcount[p] -= 1
            if self.refcount[p] == 0:
                self.free.append(p)

    @staticmethod
    def bytes_per_page(num_layers, page_size, hkv, head_dim, dtype_bytes=2) -> int:
        return 2 * num_layers * page_size * hkv * head_dim * dtype_bytes


class RolloutEngine:
    def __init__(self, weights: Qwen3Weights, *, max_batch: int = 256, page_size: int = 64,
                 num_pages: Optional[int] = None, kv_fraction: float = 0.35, max_seq_len: int = 32768,
                 split_kv_min: int = 2048):
        self.w = weights
        c = weights.cfg
        self.cfg = c
        self.dev = weights.device
        self.hq, self.hkv, self.D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        self.eps = c.rms_norm_eps
        self.max_batch = max_batch
        self.page_size = page_size
        self.max_pages_per_seq = (max_seq_len + page_size - 1) // page_size
        self.split_kv_min = split_kv_min
        self.kv_fraction = kv_fraction
        self._num_pages = num_pages
        self._cache: Optional[PagedKVCache] = None
        self.cos, self.sin = ref.rope_tables(c.max_position_embeddings, self.D, c.rope_theta, self.dev)
        self._step = 0
        self._prefix: Dict[object, tuple] = {}

    # ------------------------------------------------------------------ KV pool
    def kv_bytes_per_token(self) -> int:
        return PagedKVCache.bytes_per_page(self.cfg.num_hidden_layers, 1, self.hkv, self.D,
                                           self.w.dtype.itemsize)

    @property
    def cache(self) -> PagedKVCache:
        """The paged KV pool, allocated on first use: ``num_pages`` when given,
        else ``kv_fraction`` of the HBM free at that moment."""
        if self._cache is None:
            self.ensure_cache()
        return self._cache

    def ensure_cache(self, num_pages: Optional[int] = None) -> PagedKVCache:
        c = self.cfg
        want = num_pages or self._num_pages
        if self._cache is not None and (want is None or self._cache.num_pages >= want):
            return self._cache
        self._cache = None
        if want is None:
            per = PagedKVCache.bytes_per_page(c.num_hidden_layers, self.page_size, self.hkv, self.D)
            if self.dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(self.dev)
                free += torch.cuda.memory_reserved(self.dev) - torch.cuda.memory_allocated(self.dev)
                want = max(16, int(free * self.kv_fraction) // per)
            else:
                want = max(16, (256 << 20) // per)
        self._cache = PagedKVCache(c.num_hidden_layers, want, self.page_size, self.hkv, self.D, self.dev,
                                   self.w.dtype)
        return self._cache

    def release_cache(self) -> None:
        """Free the KV pool (it is re-allocated on next use); for phases of a
        training step that need the HBM back."""
        self._cache = None

    # ------------------------------------------------------------------ model
    def _forward(self, seqs: List[_Seq], fresh: bool, want_logits: bool = True):
        """Feed each sequence's pending tokens; returns last-token logits [B, V]."""
        dev = self.dev
        toks, pos, slots, q_start, lens = [], [], [], [0], []
        for s in seqs:
            n = len(s.pending)
            toks.extend(s.pending)
            for j in range(n):
                p = s.length + j
                pos.append(p)
                slots.append(s.pages[p // self.page_size] * self.page_size + p % self.page_size)
            q_start.append(q_start[-1] + n)
            lens.append(s.length + n)
        T = len(toks)
        ids = torch.tensor(toks, dtype=torch.long, device=dev)
        pos_t = torch.tensor(pos, dtype=torch.int32, device=dev)
        slots_t = torch.tensor(slots, dtype=torch.int32, device=dev)
        qs_t = torch.tensor(q_start, dtype=torch.int32, device=dev)
        lens_t = torch.tensor(lens, dtype=torch.int32, device=dev)
        max_q = max(len(s.pending) for s in seqs)
        bt = torch.zeros(len(seqs), self.max_pages_per_seq, dtype=torch.int32)
        for i, s in enumerate(seqs):
            bt[i, : len(s.pages)] = torch.tensor(s.pages, dtype=torch.int32)
        bt = bt.to(dev)
        max_len = max(lens)
        nsplit = max(1, min(16, max_len // self.split_kv_min)) if max_q == 1 else 1
        part_o = part_ml = None
        if nsplit > 1 and dev.type == "cuda":
            part_o = torch.empty(nsplit * T * self.hq * self.D, dtype=torch.float32, device=dev)
            part_ml = torch.empty(nsplit * T * self.hq * 2, dtype=torch.float32, device=dev)
        qd, kd = self.hq * self.D, self.hkv * self.D
        x = ops.embed_fwd(ids, self.w.views(0)["embed"])
        scale = 1.0 / math.sqrt(self.D)
        for li in range(self.cfg.num_hidden_layers):
            W = self.w.views(li + 1)
            hn = ops.rmsnorm_fwd(x, W["ln1"], self.eps)
            qkv = ops.mm(hn, W["qkv"])
            qk = ops.qk_norm_rope_fwd(qkv, W["q_norm"], W["k_norm"], pos_t, self.cos, self.sin,
                                      self.hq, self.hkv, self.eps)
            q = qk[:, :qd].view(T, self.hq, self.D)
            k = qk[:, qd:].view(T, self.hkv, self.D)
            v = qkv[:, qd + kd:].view(T, self.hkv, self.D)
            self._kv_append(k, v, slots_t, li)
            if fresh:
                o, _ = attn.attn_fwd(q, k, v, qs_t, max_q, scale)
            else:
                o = self._paged_attention(q, li, bt, lens_t, qs_t, max_q, scale, nsplit, part_o, part_ml)
            x = ops.mm(o.reshape(T, qd), W["o"], residual=x)
            hn2 = ops.rmsnorm_fwd(x, W["ln2"], self.eps)
            a = ops.swiglu_fwd(ops.mm(hn2, W["gate_up"]))
            x = ops.mm(a, W["down"], residual=x)
        for s in seqs:
            s.length += len(s.pending)
            s.pending = []
        if not want_logits:
            return None
        last = qs_t[1:] - 1
        hl = ops.rmsnorm_fwd(x.index_select(0, last), self.w.views(self.w.num_units - 1)["norm"], self.eps)
        return ops.mm(hl, self.w.lm_head_weight())

    def _kv_append(self, k, v, slots, li):
        if k.is_cuda:
            ops.native().kv_append(k, v, slots, self.cache.k[li], self.cache.v[li])
        else:
            self.cache.k[li][slots.long()] = k
            self.cache.v[li][slots.long()] = v

    def _paged_attention(self, q, li, bt, lens, qs, max_q, scale, nsplit, part_o, part_ml):
        T = q.shape[0]
        if q.is_cuda:
            out = torch.empty(T, self.hq, self.D, dtype=q.dtype, device=q.device)
            ops.native().paged_attention(q, self.cache.k[li], self.cache.v[li], bt, lens, qs, int(max_q),
                                         self.page_size, float(scale), int(nsplit), out, part_o, part_ml)
            return out
        return paged_attention_reference(q, self.cache.k[li], self.cache.v[li], bt, lens, qs,
                                         self.page_size, scale)

    def _sample(self, logits, temperature, top_p, seed):
        B = logits.shape[0]
        self._step += 1
        if logits.is_cuda:
            tok = torch.empty(B, dtype=torch.long, device=logits.device)
            lp = torch.empty(B, dtype=torch.float32, device=logits.device)
            ops.native().sample_tokens(logits, float(temperature), float(top_p), int(seed) & 0x7FFFFFFF,
                                       self._step, tok, lp)
            return tok, lp
        return sample_reference(logits, temperature, top_p, seed * 1000003 + self._step)

    # ------------------------------------------------------------------ public
    @torch.no_grad()
    def generate(self, requests: List[GenRequest], *, temperature: float = 1.0, top_p: float = 1.0,
                 eos_ids: Sequence[int] = (), seed: int = 0) -> List[GenResult]:
        """Continuous-batching generation of every request."""
        waiting = list(requests)
        active: List[_Seq] = []
        done: Dict[int, GenResult] = {}
        eos = set(int(e) for e in eos_ids)
        while waiting or active:
            admitted = self._admit(waiting, active)
            if admitted:
                fresh = [s for s in admitted if s.length == 0]
                extend = [s for s in admitted if s.length > 0]
                for group, is_fresh in ((fresh, True), (extend, False)):
                    if not group:
                        continue
                    logits = self._forward(group, fresh=is_fresh)
                    self._emit(group, logits, temperature, top_p, seed, eos)
            if not active:
                if waiting:
                    raise RuntimeError("KV cache too small for the next request")
                break
            decoding = [s for s in active if s.pending and s not in admitted]
            if decoding:
                logits = self._forward(decoding, fresh=False)
                self._emit(decoding, logits, temperature, top_p, seed, eos)
            for s in list(active):
                if s.done:
                    active.remove(s)
                    self.cache.release(s.pages)
                    done[s.req.rid] = GenResult(s.req.rid, s.out, s.logps, s.reason)
        self._prefix.clear()
        return [done[r.rid] for r in requests]

    def _emit(self, seqs, logits, temperature, top_p, seed, eos):
        tok, lp = self._sample(logits, temperature, top_p, seed)
        tok_l = tok.tolist()
        lp_l = lp.tolist()
        for s, t, l in zip(seqs, tok_l, lp_l):
            s.out.append(int(t))
            s.logps.append(float(l))
            if int(t) in eos:
                s.done, s.reason = True, "stop"
            elif len(s.out) >= s.req.max_new_tokens:
                s.done, s.reason = True, "length"
            else:
                s.pending = [int(t)]
                need = (s.length + 1 + self.page_size - 1) // self.page_size
                if need > len(s.pages):
                    p = self.cache.alloc(need - len(s.pages))
                    if p is None:       # out of pages: stop this sequence
                        s.done, s.reason = True, "kv_full"
                    else:
                        s.pages.extend(p)

    def _admit(self, waiting: List[GenRequest], active: List[_Seq]) -> List[_Seq]:
        out = []
        while waiting and len(active) < self.max_batch:
            r = waiting[0]
            n = len(r.prompt)
            need = (n + 1 + self.page_size - 1) // self.page_size
            shared: List[int] = []
            length = 0
            if r.share_key is not None and r.share_key in self._prefix:
                pages, plen = self._prefix[r.share_key]
                # share only full pages and keep >= 1 prompt token to feed
                full = min(plen - 1, n - 1) // self.page_size
                shared = pages[:full]
                length = full * self.page_size
            own = self.cache.alloc(need - len(shared))
            if own is None:
                break
            if shared:
                self.cache.retain(shared)
            waiting.pop(0)
            s = _Seq(r, shared + own, len(shared), length, list(r.prompt[length:]))
            if r.share_key is not None and r.share_key not in self._prefix:
                self._prefix[r.share_key] = (s.pages, n)
            active.append(s)
            out.append(s)
        # sequences reusing a prefix are prefilled after their owners: generate()
        # runs the fresh (owner) group before the extend group
        return out


# ---------------------------------------------------------------------- CPU refs
def paged_attention_reference(q, kc, vc, bt, lens, qs, page_size, scale):
    """fp32 PyTorch definition of the paged attention (CPU path and test oracle)."""
    T, hq, D = q.shape
    hkv = kc.shape[1]
    out = torch.empty_like(q)
    qs_l, lens_l = qs.tolist(), lens.tolist()
    for i in range(len(lens_l)):
        a, b = qs_l[i], qs_l[i + 1]
        L = lens_l[i]
        npg = (L + page_size - 1) // page_size
        pages = bt[i, :npg].long()
        slots = (pages[:, None] * page_size + torch.arange(page_size, device=q.device)[None]).reshape(-1)[:L]
        K = kc[slots].float().repeat_interleave(hq // hkv, 1)   # [L, hq, D]
        Vv = vc[slots].float().repeat_interleave(hq // hkv, 1)
        qq = q[a:b].float()                                      # [n, hq, D]
        s = torch.einsum("nhd,lhd->hnl", qq, K) * scale
        n = b - a
        qpos = torch.arange(L - n, L, device=q.device)[:, None]
        mask = torch.arange(L, device=q.device)[None, :] <= qpos
        s = s.masked_fill(~mask[None], float("-inf"))
        out[a:b] = torch.einsum("hnl,lhd->nhd", s.softmax(-1), Vv).to(q.dtype)
    return out


def sample_reference(logits, temperature, top_p, seed):
    """Torch sampler with the same semantics (CPU path)."""
    g = torch.Generator(device=logits.device)
    g.manual_seed(int(seed) & 0x7FFFFFFF)
    z = logits.float()
    if temperature <= 0:
        tok = z.argmax(-1)
        lp = torch.log_softmax(z, -1).gather(-1, tok[:, None])[:, 0]
        return tok, lp
    z = z / temperature
    logp = torch.log_softmax(z, -1)
    p = logp.exp()
    if top_p < 1.0:
        sp, si = p.sort(-1, descending=True)
        keep = (sp.cumsum(-1) - sp) < top_p
        mask = torch.zeros_like(p, dtype=torch.bool).scatter(-1, si, keep)
        p = torch.where(mask, p, torch.zeros_like(p))
    tok = torch.multinomial(p / p.sum(-1, keepdim=True), 1, generator=g)[:, 0]
    return tok, logp.gather(-1, tok[:, None])[:, 0]
