"""Multi-turn batched rollout with a CUDA-graph decode loop.

GRPO's rollout is a fixed set of trajectories (prompts x group) that refine
over a few turns. This module runs all of them as one batch:

* Pages for every trajectory's whole multi-turn transcript are reserved up
  front (prompt + turns x (max_new + feedback)), and trajectories of one group
  share their prompt's full pages, so no allocation happens while decoding.
* Prefill (turn 0) and the feedback "extend" chunks of later turns run through
  :class:`RolloutEngine`'s packed forward (varlen flash attention / paged
  attention with q_len > 1).
* Decoding runs a :class:`DecodeGraph`: the whole step (embedding, 40 layers,
  lm_head, sampler, bookkeeping) is captured once as a CUDA graph over
  device-resident state (current token, position, block table, active flag,
  output columns, RNG step), then replayed; the host only polls "any row still
  active?" every ``poll`` steps. Rows that sample EOS or reach their budget stop
  advancing (their writes go to a slot they own) and the loop ends early when
  all have stopped.

Sampler semantics (temperature, top-p, Gumbel-max, log-prob under the
temperature-scaled distribution) are those of :meth:`RolloutEngine._sample`.
Reference parity: the reference's per-turn HF ``generate`` loop
(kore/policy/grpo.py:2365-2500).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import torch

from .. import ops
from .rollout import GenRequest, RolloutEngine, _Seq


@dataclass
class TrajectoryOut:
    gens: List[List[int]] = field(default_factory=list)
    logps: List[List[float]] = field(default_factory=list)
    finish: List[str] = field(default_factory=list)
    contexts: List[List[int]] = field(default_factory=list)   # full transcript before each turn


class DecodeGraph:
    """One decode step for ``B`` rows over device-resident state; captured as
    a CUDA graph on first use (CUDA only; eager on CPU)."""

    def __init__(self, eng: RolloutEngine, B: int, max_new: int, *, nsplit: int = 4,
                 temperature: float = 1.0, top_p: float = 1.0, seed: int = 0, eos_ids: Sequence[int] = ()):
        dev = eng.dev
        self.eng, self.B, self.max_new = eng, B, max_new
        self.temperature, self.top_p, self.seed = float(temperature), float(top_p), int(seed) & 0x7FFFFFFF
        self.nsplit = nsplit if dev.type == "cuda" else 1
        i32 = dict(dtype=torch.int32, device=dev)
        self.tok = torch.zeros(B, dtype=torch.long, device=dev)
        self.pos = torch.zeros(B, **i32)
        self.bt = torch.zeros(B, eng.max_pages_per_seq, **i32)
        self.active = torch.zeros(B, dtype=torch.bool, device=dev)
        self.budget = torch.zeros(B, **i32)         # tokens this row may still emit in the turn
        self.nout = torch.zeros(B, **i32)
        self.col = torch.zeros(1, dtype=torch.long, device=dev)
        self.rng_step = torch.zeros(1, **i32)
        self.out_tok = torch.zeros(B, max_new, dtype=torch.long, device=dev)
        self.out_lp = torch.zeros(B, max_new, dtype=torch.float32, device=dev)
        self.qs = torch.arange(B + 1, **i32)
        self.eos = torch.tensor(sorted(set(int(e) for e in eos_ids)) or [-1], dtype=torch.long, device=dev)
        T, hq, D = B, eng.hq, eng.D
        self.part_o = self.part_ml = None
        if self.nsplit > 1:
            self.part_o = torch.empty(self.nsplit * T * hq * D, dtype=torch.float32, device=dev)
            self.part_ml = torch.empty(self.nsplit * T * hq * 2, dtype=torch.float32, device=dev)
        self.graph = None
        self._new_tok = torch.zeros(B, dtype=torch.long, device=dev)
        self._new_lp = torch.zeros(B, dtype=torch.float32, device=dev)

    # -------------------------------------------------------------- one step
    def _body(self) -> None:
        eng, c = self.eng, self.eng.cfg
        ps = eng.page_size
        B = self.B
        pos = self.pos
        page = self.bt.gather(1, torch.div(pos, ps, rounding_mode="floor").long().unsqueeze(1)).squeeze(1)
        slots = page * ps + torch.remainder(pos, ps)
        lens = pos + 1
        qd, kd = eng.hq * eng.D, eng.hkv * eng.D
        x = ops.embed_fwd(self.tok, eng.w.views(0)["embed"])
        scale = 1.0 / math.sqrt(eng.D)
        for li in range(c.num_hidden_layers):
            W = eng.w.views(li + 1)
            hn = ops.rmsnorm_fwd(x, W["ln1"], eng.eps)
            qkv = ops.mm(hn, W["qkv"])
            qk = ops.qk_norm_rope_fwd(qkv, W["q_norm"], W["k_norm"], pos, eng.cos, eng.sin,
                                      eng.hq, eng.hkv, eng.eps)
            q = qk[:, :qd].view(B, eng.hq, eng.D)
            k = qk[:, qd:].view(B, eng.hkv, eng.D)
            v = qkv[:, qd + kd:].view(B, eng.hkv, eng.D)
            eng._kv_append(k, v, slots, li)
            o = eng._paged_attention(q, li, self.bt, lens, self.qs, 1, scale, self.nsplit, self.part_o,
                                     self.part_ml)
            x = ops.mm(o.reshape(B, qd), W["o"], residual=x)
            hn2 = ops.rmsnorm_fwd(x, W["ln2"], eng.eps)
            a = ops.swiglu_fwd(ops.mm(hn2, W["gate_up"]))
            x = ops.mm(a, W["down"], residual=x)
        hl = ops.rmsnorm_fwd(x, eng.w.views(eng.w.num_units - 1)["norm"], eng.eps)
        logits = ops.mm(hl, eng.w.lm_head_weight())
        if logits.is_cuda:
            ops.native().sample_tokens(logits, self.temperature, self.top_p, self.seed, 0, self._new_tok,
                                       self._new_lp, self.rng_step)
        else:
            from .rollout import sample_reference
            t, l = sample_reference(logits, self.temperature, self.top_p,
                                    self.seed * 1000003 + int(self.rng_step.item()))
            self._new_tok.copy_(t)
            self._new_lp.copy_(l)
        act = self.active
        self.out_tok.index_copy_(1, self.col, torch.where(act, self._new_tok, torch.zeros_like(self._new_tok))
                                 .unsqueeze(1))
        self.out_lp.index_copy_(1, self.col, torch.where(act, self._new_lp, torch.zeros_like(self._new_lp))
                                .unsqueeze(1))
        ai = act.to(torch.int32)
        self.nout.add_(ai)
        self.pos.add_(ai)
        self.tok.copy_(torch.where(act, self._new_tok, self.tok))
        stop = (self._new_tok.unsqueeze(1) == self.eos.unsqueeze(0)).any(1) | (self.nout >= self.budget)
        self.active.logical_and_(~stop)
        self.col.add_(1)
        self.rng_step.add_(1)

    def step(self) -> None:
        if self.eng.dev.type != "cuda":
            self._body()
            return
        if self.graph is None:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                # warm-up launch (kernel attributes, allocator pool) outside capture,
                # on a copy of the state so the real step is not consumed
                saved = [t.clone() for t in self._state()]
                self._body()
                for t, v in zip(self._state(), saved):
                    t.copy_(v)
            torch.cuda.current_stream().wait_stream(s)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._body()
        self.graph.replay()

    def _state(self):
        return [self.tok, self.pos, self.active, self.nout, self.col, self.rng_step, self.out_tok, self.out_lp]


class MultiTurnRollout:
    """Rolls a fixed set of trajectories through ``num_turns`` turns."""

    def __init__(self, eng: RolloutEngine, *, poll: int = 128, nsplit: int = 4):
        self.eng = eng
        self.poll = poll
        self.nsplit = nsplit

    @torch.no_grad()
    def run(self, prompts: List[List[int]], *, num_turns: int, max_new: int,
            feedback: Callable[[int, int, List[int]], List[int]], share_keys: Optional[list] = None,
            max_feedback: int = 256, temperature: float = 1.0, top_p: float = 1.0,
            eos_ids: Sequence[int] = (), seed: int = 0,
            on_turn: Optional[Callable[[int, List[TrajectoryOut]], None]] = None) -> List[TrajectoryOut]:
        """``feedback(turn, traj, gen_tokens) -> ids`` appended after each turn
        but the last (at most ``max_feedback`` tokens). ``on_turn`` is called
        after every turn (e.g. to score it)."""
        eng = self.eng
        n = len(prompts)
        ps = eng.page_size
        cap = max(len(p) for p in prompts) + num_turns * (max_new + max_feedback) + 1
        need_pages = (cap + ps - 1) // ps
        if need_pages > eng.max_pages_per_seq:
            raise ValueError(f"transcript of {cap} tokens exceeds the engine's max_seq_len")
        if eng._cache is None and eng._num_pages is None:
            eng.ensure_cache(n * need_pages)        # exactly what this batch can use
        # ---- page reservation with prompt sharing inside a group
        seqs: List[_Seq] = []
        owners = {}
        for i, p in enumerate(prompts):
            key = share_keys[i] if share_keys is not None else None
            shared: List[int] = []
            length = 0
            if key is not None and key in owners:
                o_pages, plen = owners[key]
                full = min(plen - 1, len(p) - 1) // ps
                shared = o_pages[:full]
                length = full * ps
            own = eng.cache.alloc(need_pages - len(shared))
            if own is None:
                for s in seqs:
                    eng.cache.release(s.pages)
                raise RuntimeError(f"KV cache too small for {n} trajectories of {cap} tokens")
            if shared:
                eng.cache.retain(shared)
            s = _Seq(GenRequest(list(p), max_new, rid=i), shared + own, len(shared), length, list(p[length:]))
            if key is not None and key not in owners:
                owners[key] = (s.pages, len(p))
            seqs.append(s)
        outs = [TrajectoryOut() for _ in range(n)]
        transcripts = [list(p) for p in prompts]
        g = DecodeGraph(eng, n, max_new, nsplit=self.nsplit, temperature=temperature, top_p=top_p,
                        seed=seed, eos_ids=eos_ids)
        g.bt.zero_()
        for i, s in enumerate(seqs):
            g.bt[i, : len(s.pages)] = torch.tensor(s.pages, dtype=torch.int32)
        try:
            for turn in range(num_turns):
                for i in range(n):
                    outs[i].contexts.append(list(transcripts[i]))
                # ---- prefill / extend: owners (fresh) first, then everything with history
                fresh = [s for s in seqs if s.length == 0]
                rest = [s for s in seqs if s.length > 0]
                first_tok = torch.zeros(n, dtype=torch.long, device=eng.dev)
                first_lp = torch.zeros(n, dtype=torch.float32, device=eng.dev)
                for group, is_fresh in ((fresh, True), (rest, False)):
                    if not group:
                        continue
                    logits = eng._forward(group, fresh=is_fresh)
                    t, l = eng._sample(logits, temperature, top_p, seed * 7919 + turn)
                    idx = torch.tensor([s.req.rid for s in group], dtype=torch.long, device=eng.dev)
                    first_tok.index_copy_(0, idx, t)
                    first_lp.index_copy_(0, idx, l)
                # ---- decode state for this turn
                g.pos.copy_(torch.tensor([s.length for s in seqs], dtype=torch.int32))
                g.tok.copy_(first_tok)
                g.out_tok.zero_()
                g.out_lp.zero_()
                g.out_tok[:, 0] = first_tok
                g.out_lp[:, 0] = first_lp
                g.nout.fill_(1)
                g.budget.fill_(max_new)
                g.col.fill_(1)
                g.active.copy_(~torch.isin(first_tok, g.eos) & (g.nout < g.budget))
                steps = 1
                while steps < max_new:
                    burst = min(self.poll, max_new - steps)
                    for _ in range(burst):
                        g.step()
                    steps += burst
                    if not bool(g.active.any()):
                        break
                nout = g.nout.tolist()
                toks = g.out_tok.tolist()
                lps = g.out_lp.tolist()
                pos_after = g.pos.tolist()
                for i, s in enumerate(seqs):
                    k = nout[i]
                    gen, lp = toks[i][:k], lps[i][:k]
                    outs[i].gens.append(gen)
                    outs[i].logps.append(lp)
                    outs[i].finish.append("stop" if gen and int(gen[-1]) in set(int(e) for e in eos_ids)
                                          else "length")
                    # the last sampled token was never fed: it heads the next extend chunk
                    s.length = pos_after[i]
                    transcripts[i] += gen
                if on_turn is not None:
                    on_turn(turn, outs)
                if turn + 1 < num_turns:
                    for i, s in enumerate(seqs):
                        fb = list(feedback(turn, i, outs[i].gens[-1]))[:max_feedback]
                        s.pending = [transcripts[i][-1]] + fb
                        transcripts[i] += fb
        finally:
            for s in seqs:
                eng.cache.release(s.pages)
        return outs
