"""Multi-turn GRPO trainer (Kevin credit + anti-collapse ladder) on the
explicit engine and the paged rollout engine.

One optimizer step:
  1. rollout: for each task group, ``num_trajectories`` trajectories refine
     their answer over ``num_turns`` turns (serial refinement); each turn's
     context is the transcript so far plus the environment's feedback. The
     rollout engine generates every trajectory of the group in one continuous
     batch, sharing the prompt's KV pages inside the group. Trajectories are
     split over ranks with a strided slice (replicated rollout on every rank);
  2. credit: per-turn Kevin returns (correctness-gated, gamma look-ahead,
     optional potential-based shaping), infra turns dropped; group-relative
     AVSPO advantages over the group's per-turn samples gathered from all
     ranks; StarPO-S / DAPO dynamic sampling keep the informative groups;
  3. old/ref log-probs: old = the sampler's temperature-scaled log-probs of
     the generated tokens (token mean), ref = a frozen reference model
     forward (token mean);
  4. update: global token-mean clip-higher surrogate + k3 KL anchor, as
     per-token coefficients into the engine's two-phase head (packed
     micro-batches, no autograd graph), one AdamW step (sharded over ranks),
     then the weight sync back to the rollout engine (free on one GPU: the
     engine reads the trainer's buffers).

Behavioural parity: kore/policy/grpo.py:565-2331 (train_grpo, Kevin credit,
_accumulate_grpo_grads, the distributed loop).
"""
from __future__ import annotations

import json
import math
import os
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch

from ..env.base import RolloutEnv, SyntheticRewardEnv, TurnResult
from ..obs import configure, get_logger
from ..parallel.dist import DistContext, get_context, init_distributed
from . import rl_math as M
from .configs import GRPOConfig, grpo_config_from_dict

log = get_logger("policy.grpo")


@dataclass
class Trajectory:
    traj: int
    contexts: List[List[int]] = field(default_factory=list)   # prompt ids of each turn
    gens: List[List[int]] = field(default_factory=list)       # generated ids of each turn
    gen_logps: List[List[float]] = field(default_factory=list)
    results: List[TurnResult] = field(default_factory=list)
    finish: List[str] = field(default_factory=list)


@dataclass
class TrainSample:
    ids: List[int]          # context + generation
    n_ctx: int
    ret: float
    adv: float = 0.0
    old_logp: Optional[float] = None
    ref_logp: Optional[float] = None
    overlong: bool = False
    row: Optional[tuple] = None     # (group, trajectory): samples of one trajectory share a packed row
    turn: int = 0

    @property
    def n_gen(self) -> int:
        return len(self.ids) - self.n_ctx


class GRPOTrainer:
    """GRPO over a :class:`CausalLMTrainer`-style engine/optimizer pair."""

    def __init__(self, config: GRPOConfig, *, weights=None, ref_weights=None, env: Optional[RolloutEnv] = None,
                 ctx: Optional[DistContext] = None, tokenizer=None, model_cfg=None,
                 rollout_kwargs: Optional[dict] = None):
        from ..engine.qwen3_engine import Qwen3Engine
        from ..engine.rollout import RolloutEngine
        from ..engine.trainer import CausalLMTrainer
        from ..models import Qwen3Config, Qwen3Weights
        self.cfg = config
        self.ctx = ctx or get_context()
        self.env = env or SyntheticRewardEnv(seed=config.seed)
        self.tok = tokenizer
        if weights is None:
            mc = model_cfg or Qwen3Config()
            dtype = torch.bfloat16 if (config.bf16 and self.ctx.device.type == "cuda") else torch.float32
            weights = Qwen3Weights(mc, device=self.ctx.device, dtype=dtype, seed=config.seed,
                                   pad_multiple=128 * max(1, self.ctx.world))
        self.trainer = CausalLMTrainer(weights.cfg, self.ctx, lr=config.learning_rate,
                                       max_grad_norm=config.max_grad_norm, seed=config.seed,
                                       schedule=config.lr_scheduler_type,
                                       warmup_steps=int(config.warmup_ratio * config.total_steps),
                                       total_steps=config.total_steps, weights=weights,
                                       comm=getattr(config, "comm", "nccl"))
        self.trainer.eng.temperature = config.temperature
        # the trainer may have moved the weights (e.g. into the symmetric heap of
        # the fused optimizer): rollout and reference read the trainer's copy
        self.w = weights = self.trainer.w
        self.ref_w, self.ref_stream = None, None
        self.ref_placement = "none"
        if ref_weights is not None or config.ref_anchor_coef:
            self.ref_w, self.ref_placement = self._build_ref(ref_weights, getattr(config, "ref_placement", "auto"))
        self.ref_eng = (Qwen3Engine(self.ref_w, allocate_grads=False, temperature=config.temperature)
                        if self.ref_w is not None else None)
        if self.ref_eng is not None and self.ref_stream is not None:
            self.ref_eng.param_hook = self.ref_stream
        rk = dict(max_batch=config.rollout_max_batch, page_size=min(config.kv_page_size, 128),
                  kv_fraction=config.kv_cache_fraction)
        rk.update(rollout_kwargs or {})
        self.rollout = RolloutEngine(self.w, **rk)
        self.step_idx = 0
        self.controller = (M.DynamicStepController(config.min_steps, config.total_steps,
                                                   config.plateau_patience, config.plateau_min_delta)
                           if config.adaptive_steps else None)
        from .grpo_hooks import CurriculumHook, SearchDistill, ValuePrefilter
        self.curriculum = CurriculumHook(self) if config.coevolve else None
        self.prefilter = ValuePrefilter(self) if config.value_prefilter else None
        self.search_hook = SearchDistill(self) if config.use_search else None
        self.eos = []
        if tokenizer is not None:
            from ..data.tokenizer import eos_ids
            self.eos = eos_ids(tokenizer)

    def _build_ref(self, ref_weights, mode: str):
        """The frozen KL reference: resident, or its decoder layers streamed
        from pinned host memory (one GPU) / sharded and all-gathered per layer
        (several ranks). ``auto`` keeps it resident only when a second copy of
        the weights leaves 40 GB of HBM for the rollout and activations."""
        from ..engine.frozen_stream import FrozenLayerStream
        from ..models import Qwen3Weights
        src = ref_weights if ref_weights is not None else self.w
        if mode == "auto":
            mode = "resident"
            if self.ctx.world > 1:
                mode = "shard"
            elif src.device.type == "cuda":
                free, _ = torch.cuda.mem_get_info(src.device)
                need = sum(b.numel() * b.element_size() for b in src.bufs if b is not None)
                mode = "host" if free < need + 40e9 else "resident"
        if mode == "resident":
            return (ref_weights if ref_weights is not None else self.w.clone()), mode
        ref = Qwen3Weights(src.cfg, device=src.device, dtype=src.dtype, allocate=False,
                           pad_multiple=src.pad_multiple, ep=src.ep)
        last = src.num_units - 1
        ref.bufs = [src.bufs[u].clone() if u in (0, last) else None for u in range(src.num_units)]
        ref.expert_bufs = {u: b.clone() for u, b in src.expert_bufs.items()}
        self.ref_stream = FrozenLayerStream(ref, source=mode, ctx=self.ctx, layers_from=src)
        return ref, mode

    # ------------------------------------------------------------ rollout
    def _decode(self, ids: Sequence[int]) -> str:
        if self.tok is None:
            return ""
        return self.tok.decode(list(ids))

    def _initial_context(self, task) -> List[int]:
        if isinstance(self.env, SyntheticRewardEnv):
            return self.env.prompt_ids(task)
        from ..data.tokenizer import render_chat
        ids, _ = render_chat(self.tok, self.env.prompt_messages(task), add_generation_prompt=True)
        return ids[-self.cfg.max_prompt_length:]

    def _feedback_ids(self, task, tr: TurnResult, turn: int, traj: int) -> List[int]:
        if isinstance(self.env, SyntheticRewardEnv):
            return self.env.feedback_ids(task, turn, traj)
        from ..data.tokenizer import render_chat
        ids, _ = render_chat(self.tok, [{"role": "user", "content": f"Verifier feedback:\n{tr.feedback}"}],
                             add_generation_prompt=True)
        return ids

    def rollout_group(self, task, traj_ids: Sequence[int], *, max_new_tokens: Optional[int] = None
                      ) -> List[Trajectory]:
        cfg = self.cfg
        max_new = max_new_tokens or cfg.max_response_length
        base = self._initial_context(task)
        trajs = [Trajectory(t) for t in traj_ids]
        ctxs = [list(base) for _ in trajs]
        ncand = self.prefilter.n if self.prefilter is not None else 1
        for turn in range(cfg.num_turns):
            from ..engine.rollout import GenRequest
            reqs = []
            for i, (tr, c) in enumerate(zip(trajs, ctxs)):
                c = c[-cfg.max_prompt_length:]
                ctxs[i] = c
                key = (task, "t0") if (turn == 0 and ncand == 1) else ((task, turn, i) if ncand > 1 else None)
                for j in range(ncand):
                    reqs.append(GenRequest(prompt=c, max_new_tokens=max_new, rid=i * ncand + j, share_key=key))
            outs = self.rollout.generate(reqs, temperature=cfg.temperature, top_p=cfg.top_p,
                                         eos_ids=self.eos, seed=cfg.seed * 1000003 + self.step_idx * 97 + turn)
            for i, tr in enumerate(trajs):
                cands = outs[i * ncand:(i + 1) * ncand]
                if ncand == 1:
                    o = cands[0]
                    res = self.env.step(task, self._decode(o.tokens), turn, tr.traj, tr.results)
                else:   # value prefilter: verify only the value model's top-k candidates
                    from .format import parse_response
                    texts = [self._decode(o.tokens) for o in cands]
                    pick = self.prefilter.pick([parse_response(t).get("kernel", "") for t in texts])
                    best = None
                    for j in pick:
                        r = self.env.step(task, texts[j], turn, tr.traj, tr.results)
                        if best is None or (r.correct, r.reward) > (best[1].correct, best[1].reward):
                            best = (j, r)
                    o, res = cands[best[0]], best[1]
                tr.contexts.append(list(ctxs[i]))
                tr.gens.append(list(o.tokens))
                tr.gen_logps.append(list(o.logps))
                tr.finish.append(o.finish_reason)
                tr.results.append(res)
                ctxs[i] = ctxs[i] + list(o.tokens) + self._feedback_ids(task, res, turn, tr.traj)
        return trajs

    def rollout_batch(self, tasks: Sequence[Any], traj_ids: Sequence[int], *,
                      max_new_tokens: Optional[int] = None) -> List[List[Trajectory]]:
        """Every group of the step (``tasks`` x ``traj_ids``) in one multi-turn
        batch on the CUDA-graph decode loop; groups share their prompt's KV pages.
        Same transcripts as :meth:`rollout_group` while they fit ``max_prompt_length``."""
        from ..engine.multiturn import MultiTurnRollout
        cfg = self.cfg
        max_new = max_new_tokens or cfg.max_response_length
        G = len(traj_ids)
        prompts, keys = [], []
        for gi, task in enumerate(tasks):
            base = self._initial_context(task)[-cfg.max_prompt_length:]
            for _ in traj_ids:
                prompts.append(list(base))
                keys.append(gi)
        groups = [[Trajectory(t) for t in traj_ids] for _ in tasks]
        flat = [tr for g in groups for tr in g]

        def on_turn(turn, outs):
            for i, (o, tr) in enumerate(zip(outs, flat)):
                tr.results.append(self.env.step(tasks[i // G], self._decode(o.gens[-1]), turn, tr.traj,
                                                tr.results))

        def feedback(turn, i, gen):
            tr = flat[i]
            return self._feedback_ids(tasks[i // G], tr.results[-1], turn, tr.traj)

        fb_cap = cfg.max_feedback_tokens
        if isinstance(self.env, SyntheticRewardEnv):
            fb_cap = min(fb_cap, self.env.feedback_len)
        if self._use_tp():
            outs = self._rollout_tp(prompts, max_new, fb_cap, feedback, on_turn)
            for o, tr in zip(outs, flat):
                tr.contexts, tr.gens, tr.gen_logps, tr.finish = o.contexts, o.gens, o.logps, o.finish
            return groups
        outs = MultiTurnRollout(self.rollout).run(
            prompts, num_turns=cfg.num_turns, max_new=max_new, feedback=feedback, share_keys=keys,
            max_feedback=fb_cap, temperature=cfg.temperature, top_p=cfg.top_p,
            eos_ids=self.eos, seed=cfg.seed * 1000003 + self.step_idx * 97, on_turn=on_turn)
        for o, tr in zip(outs, flat):
            tr.contexts, tr.gens, tr.gen_logps, tr.finish = o.contexts, o.gens, o.logps, o.finish
        return groups

    def _use_tp(self) -> bool:
        return getattr(self.cfg, "rollout_parallel", "replica") == "tp" and self.ctx.world > 1

    def _rollout_tp(self, prompts, max_new: int, fb_cap: int, feedback, on_turn):
        """Multi-turn rollout on the tensor-parallel engine: every rank holds
        1/world of each layer's heads and FFN columns and all ranks decode all
        ranks' rows together (AG->GEMM / GEMM->RS over peer memory). Turn t+1
        extends the cache by the last sampled token and the feedback only."""
        from ..engine.multiturn import TrajectoryOut
        from ..parallel.tp import TPRolloutEngine
        cfg = self.cfg
        n = len(prompts)
        cap = max(len(p) for p in prompts) + cfg.num_turns * (max_new + fb_cap) + 1
        cap = self.ctx.all_gather_object(cap) if self.ctx.world > 1 else [cap]
        cap = max(cap)
        if getattr(self, "tp", None) is None or self.tp.S < n or self.tp.max_seq_len < cap:
            self.tp = None
            if self.ctx.device.type == "cuda":
                torch.cuda.empty_cache()
            self.tp = TPRolloutEngine(self.w, self.ctx, max_rows=4096, max_seqs=n, max_seq_len=cap)
        tp = self.tp
        tp.reset()
        outs = [TrajectoryOut() for _ in range(n)]
        ctxs = [list(p) for p in prompts]
        pending = [list(p) for p in prompts]
        eos = set(int(e) for e in self.eos)
        for turn in range(cfg.num_turns):
            for i in range(n):
                outs[i].contexts.append(list(ctxs[i]))
            toks, lps = tp.generate(pending, max_new, temperature=cfg.temperature, top_p=cfg.top_p,
                                    eos_ids=self.eos, seed=cfg.seed * 1000003 + self.step_idx * 97 + turn)
            for i in range(n):
                outs[i].gens.append(toks[i])
                outs[i].logps.append(lps[i])
                outs[i].finish.append("stop" if toks[i] and int(toks[i][-1]) in eos else "length")
                ctxs[i] += toks[i]
            if on_turn is not None:
                on_turn(turn, outs)
            if turn + 1 < cfg.num_turns:
                for i in range(n):
                    fb = list(feedback(turn, i, toks[i]))[:fb_cap]
                    ctxs[i] += fb
                    pending[i] = ([toks[i][-1]] if toks[i] else []) + fb
        tp.release_cache()
        return outs

    def memory_plan(self, trajectories: int, transcript: int) -> Dict[str, object]:
        """What leaves HBM during the rollout and reference phases of a step.

        The KV cache of ``trajectories`` transcripts of ``transcript`` tokens
        must fit next to the weights. In that order, and only as far as needed:
        (1) the gradient buffers are dropped (they are zeroed at the start of
        every update anyway, so nothing is copied) when they are plain tensors;
        (2) optimizer state tensors (second moments first, then first moments,
        then the fp32 master) are parked in host memory, which is bounded too.
        ``ref``: a resident frozen reference leaves HBM for the update when the
        update's activations would not fit. ``offload_state`` = always parks
        all optimizer state; never parks nothing."""
        from ..engine.offload import optimizer_slots, slots_bytes
        mode = self.cfg.offload_state
        dev = self.ctx.device
        none = {"grads": False, "opt": [], "ref": False}
        if mode == "never" or dev.type != "cuda":
            return none
        slots = optimizer_slots(self.trainer.opt)
        order = sorted(slots, key=lambda s: {"v": 0, "m": 1, "master": 2}.get(self._slot_kind(s), 3))
        if mode == "always":
            return {"grads": self.trainer.heap is None, "opt": order,
                    "ref": self.ref_w is not None and self.ref_stream is None}
        torch.cuda.empty_cache()                 # count only memory a fresh allocation can get
        free, _ = torch.cuda.mem_get_info(dev)
        kv = trajectories * transcript * self.rollout.kv_bytes_per_token()
        if self._use_tp() and getattr(self, "tp", None) is None:
            # the tensor-parallel engine is built at the first rollout: its head /
            # FFN slice of every layer and its peer-memory buffers
            W, H = self.ctx.world, self.w.cfg.hidden_size
            layers = sum(self.w.padded_numel(u) for u in range(1, self.w.num_units - 1))
            kv += layers * 2 // W + 4096 * H * 2 * (1 + 2 * W)
        need = kv + 10e9 - free
        plan: Dict[str, object] = dict(none)
        if need > 0 and self.trainer.heap is None:
            gbytes = sum(g.numel() * g.element_size() for g in self.trainer.eng.grads if g is not None)
            plan["grads"] = True
            need -= gbytes
        picked = []
        for s in order:
            if need <= 0:
                break
            picked.append(s)
            need -= slots_bytes([s])
        if need > 0:
            raise RuntimeError(f"rollout KV cache ({kv / 1e9:.1f} GB) does not fit even with the gradients "
                               f"dropped and the optimizer state parked in host memory")
        plan["opt"] = picked
        act = 16e9 if self.trainer.eng.keep_layers == 0 else 16e9 + 40e9
        plan["ref"] = self.ref_w is not None and act > free
        return plan

    def _ref_slots(self):
        """Device tensors of the frozen reference that are parked for the update
        (its resident units; a streamed reference also frees its layer ring,
        which is refilled from its store on the next use)."""
        from ..engine.offload import weight_slots
        slots = weight_slots(self.ref_w)
        if self.ref_stream is not None:
            self.ref_stream.free_ring()
            slots = [(c, k) for c, k in slots if not (c is self.ref_w.bufs and k in self.ref_stream.store)]
        return slots

    def _slot_kind(self, slot) -> str:
        c, _ = slot
        for name in ("m", "v", "master"):
            if c is getattr(self.trainer.opt, name, None):
                return name
        return "other"

    def _drop_grads(self) -> None:
        eng = self.trainer.eng
        self._grad_shapes = [(g.numel(), g.dtype) if g is not None else None for g in eng.grads]
        eng.grads = [None] * len(eng.grads)

    def _restore_grads(self) -> None:
        eng = self.trainer.eng
        eng.grads = [None if spec is None else torch.zeros(spec[0], dtype=spec[1], device=self.ctx.device)
                     for spec in self._grad_shapes]

    def _batched_ok(self, max_new: int) -> bool:
        cfg = self.cfg
        synth = isinstance(self.env, SyntheticRewardEnv)
        longest = self.env.prompt_len if synth else cfg.max_prompt_length
        fb = min(self.env.feedback_len, cfg.max_feedback_tokens) if synth else cfg.max_feedback_tokens
        transcript = longest + cfg.num_turns * (max_new + fb)
        return (cfg.batched_rollout and transcript <= cfg.max_prompt_length + max_new
                and transcript <= self.rollout.max_pages_per_seq * self.rollout.page_size)

    # ------------------------------------------------------------ credit
    def samples_from_group(self, trajs: List[Trajectory], group: int = 0) -> List[TrainSample]:
        cfg = self.cfg
        rewards = [[r.reward for r in t.results] for t in trajs]
        correct = [[r.correct for r in t.results] for t in trajs]
        infra = [[r.infra for r in t.results] for t in trajs]
        phis = [[r.phi for r in t.results] for t in trajs] if cfg.physics_shaping_weight else None
        rets, idx = M.build_kevin_samples(rewards, correct, cfg.gamma, infra,
                                          credit_incorrect=cfg.credit_incorrect_turns,
                                          traj_phis=phis, phi_weight=cfg.physics_shaping_weight)
        out = []
        for r, (ti, tu) in zip(rets, idx):
            t = trajs[ti]
            gl = t.gen_logps[tu]
            n = len(t.gens[tu])
            if n == 0:
                continue
            over = cfg.overlong_mask and M.is_overlong(n, cfg.max_response_length, cfg.overlong_buffer_len) \
                and t.finish[tu] == "length"
            out.append(TrainSample(ids=t.contexts[tu] + t.gens[tu], n_ctx=len(t.contexts[tu]), ret=r,
                                   old_logp=sum(gl) / max(1, len(gl)), overlong=over,
                                   row=(group, t.traj), turn=tu))
        return out

    def assign_advantages(self, groups: List[List[TrainSample]]) -> List[List[TrainSample]]:
        """Cross-rank group advantages; then StarPO-S selection of groups."""
        cfg = self.cfg
        kept_idx = list(range(len(groups)))
        per_group_returns = []
        for g in groups:
            per_rank = self.ctx.all_gather_object([s.ret for s in g])
            per_group_returns.append(per_rank)
            adv = M.distributed_group_advantages(per_rank, cfg.variance_floor, cfg.avspo_virtual_k,
                                                 cfg.adv_eps)[self.ctx.rank]
            for s, a in zip(g, adv):
                s.adv = a
        if cfg.starpo_s:
            full = [M.merge_across_ranks(pr) for pr in per_group_returns]
            kept_idx = M.starpo_select_high_variance(full, cfg.starpo_keep_frac, cfg.starpo_min_std)
        return [groups[i] for i in kept_idx]

    # ------------------------------------------------------------ update
    def _rows(self, samples: List[TrainSample]) -> List[List[TrainSample]]:
        """Trajectory packing: the turn samples of one trajectory whose token
        ids extend each other form one row (the longest sample's ids), each
        turn's generated span labelled for its own sample. Causal attention
        makes every span's log-probs identical to a forward of its own sample,
        so all turns train in one forward over the transcript instead of one
        forward per turn (the reference's per-sample backward,
        kore/policy/grpo.py:613-701, recomputes each turn's whole context)."""
        if not self.cfg.pack_trajectories:
            return [[s] for s in samples]
        keyed: Dict[Any, List[TrainSample]] = {}
        order: List[Any] = []
        for i, s in enumerate(samples):
            k = s.row if s.row is not None else ("solo", i)
            if k not in keyed:
                keyed[k] = []
                order.append(k)
            keyed[k].append(s)
        rows: List[List[TrainSample]] = []
        for k in order:
            chain: List[TrainSample] = []
            for s in sorted(keyed[k], key=lambda x: len(x.ids)):
                if chain and not (len(s.ids) >= len(chain[-1].ids) and s.ids[:len(chain[-1].ids)] == chain[-1].ids):
                    rows.append(chain)
                    chain = []
                chain.append(s)
            rows.append(chain)
        return rows

    def _pack(self, rows: List[List[TrainSample]], budget: int):
        cur, n = [], 0
        for r in rows:
            L = len(r[-1].ids)
            if cur and n + L > budget:
                yield cur
                cur, n = [], 0
            cur.append(r)
            n += L
        if cur:
            yield cur

    def _batch(self, rows: List[List[TrainSample]]):
        """Packed micro-batch of rows; returns (batch, samples in order, per-token sample index)."""
        from ..engine.qwen3_engine import Batch
        dev = self.ctx.device
        seqs, masks, flat = [], [], []
        seg = []
        for r in rows:
            ids = r[-1].ids
            seqs.append(torch.tensor(ids, dtype=torch.long))
            m = torch.zeros(len(ids), dtype=torch.bool)
            sg = torch.full((len(ids),), -1, dtype=torch.long)
            for s in r:
                m[s.n_ctx: len(s.ids)] = True
                # label position j predicts token j + 1
                sg[s.n_ctx - 1: len(s.ids) - 1] = len(flat)
                flat.append(s)
            masks.append(m)
            seg.append(sg)
        b = Batch.from_sequences(seqs, masks, device=dev)
        return b, flat, torch.cat(seg).to(dev)

    @staticmethod
    def _sample_means(lp_full, seg, flat):
        sums = torch.zeros(len(flat), dtype=torch.float64, device=lp_full.device)
        sums.index_add_(0, seg.clamp_min(0), torch.where(seg >= 0, lp_full.double(),
                                                         torch.zeros_like(lp_full, dtype=torch.float64)))
        return [v / max(1, s.n_gen) for v, s in zip(sums.tolist(), flat)]

    @torch.no_grad()
    def fill_ref_logps(self, samples: List[TrainSample], budget: int):
        if self.ref_eng is None:
            return
        chunks = [self._batch(c) for c in self._pack(self._rows(samples), budget)]
        if self.ref_stream is not None:
            # streamed / gathered reference: every layer moves once for the whole step
            lps = [lp for lp, _ in self.ref_eng.token_logprobs_many([b for b, _, _ in chunks])]
        else:
            lps = [self.ref_eng.token_logprobs(b)[0] for b, _, _ in chunks]
        for (b, flat, seg), lp in zip(chunks, lps):
            for s, v in zip(flat, self._sample_means(lp, seg, flat)):
                s.ref_logp = v

    def update(self, samples: List[TrainSample], budget: int) -> Dict[str, float]:
        cfg = self.cfg
        train = [s for s in samples if not s.overlong]
        eng = self.trainer.eng
        tot = torch.tensor([float(sum(s.n_gen for s in train))], dtype=torch.float64,
                           device=self.ctx.device if self.ctx.backend == "nccl" else "cpu")
        self.ctx.all_reduce(tot)
        total_tokens = max(1.0, float(tot.item()))
        eng.zero_grad()
        loss_sum = 0.0
        kl_sum, kl_n = 0.0, 0
        trainer_old = cfg.old_logp_source == "trainer"
        for chunk in self._pack(self._rows(train), budget):
            b, flat, seg = self._batch(chunk)

            def coef_fn(lp_full, seg=seg, flat=flat):
                lps = self._sample_means(lp_full, seg, flat)
                gs = [M.GRPOSample(adv=s.adv, n_tokens=s.n_gen,
                                   old_logp=lp if trainer_old else s.old_logp,
                                   ref_logp=s.ref_logp if cfg.ref_anchor_coef else None)
                      for s, lp in zip(flat, lps)]
                loss, coefs = M.grpo_token_coefficients(gs, lps, clip_lo=cfg.clip_ratio_low,
                                                        clip_hi=cfg.clip_ratio_high,
                                                        ref_coef=cfg.ref_anchor_coef,
                                                        total_tokens=int(total_tokens))
                cvec = torch.tensor(coefs, dtype=torch.float32, device=lp_full.device)
                coef = torch.where(seg >= 0, cvec[seg.clamp_min(0)], torch.zeros_like(lp_full))
                nonlocal kl_sum, kl_n
                for s, lp in zip(flat, lps):
                    if trainer_old:
                        s.old_logp = lp
                    if s.ref_logp is not None:
                        kl_sum += M.kl_k3(lp, s.ref_logp)
                        kl_n += 1
                return coef, loss

            out = eng.forward_backward(b, coef_fn=coef_fn)
            loss_sum += float(out["loss"])
        self.trainer.opt.step()
        return {"loss": loss_sum, "kl": kl_sum / max(1, kl_n), "tokens": total_tokens}

    # ------------------------------------------------------------ step
    def train_step(self, tasks: Sequence[Any], *, max_new_tokens: Optional[int] = None,
                   micro_batch_tokens: int = 16384) -> Dict[str, float]:
        cfg = self.cfg
        t0 = time.time()
        G = cfg.num_trajectories
        W = self.ctx.world
        if G % W:
            G += W - G % W  # every rank rolls the same number of trajectories
        mine = M.rank_slice(G, self.ctx.rank, W)
        groups: List[List[TrainSample]] = []
        rewards_all: List[float] = []
        gen_tokens = 0
        traj_tokens = 0

        if self.curriculum is not None:
            tasks = self.curriculum.choose(tasks, cfg.target_groups or len(tasks))
        traj_groups: List[tuple] = []

        def roll(attempt):
            task = tasks[attempt % len(tasks)]
            if cfg.agentic:
                from .grpo_hooks import rollout_agentic
                trajs = rollout_agentic(self, task, mine, max_new_tokens or cfg.max_response_length)
            else:
                trajs = self.rollout_group(task, mine, max_new_tokens=max_new_tokens)
            traj_groups.append((task, trajs))
            nonlocal gen_tokens
            gen_tokens += sum(len(g) for t in trajs for g in t.gens)
            return self.samples_from_group(trajs, attempt), [M.kevin_trajectory_score(
                [r.reward for r in t.results], [r.correct for r in t.results]) for t in trajs]

        from ..obs import PhaseTimer
        pt = PhaseTimer()
        target = cfg.target_groups or len(tasks)
        ph = pt.phase("rollout")
        ph.__enter__()
        max_new = max_new_tokens or cfg.max_response_length
        plan = {"grads": False, "opt": [], "ref": False}
        batched = self._batched_ok(max_new) and not cfg.dynamic_sampling and not cfg.agentic \
            and self.prefilter is None
        if batched:
            from ..engine.offload import HostStash, optimizer_slots, weight_slots
            plen = self.env.prompt_len if isinstance(self.env, SyntheticRewardEnv) else cfg.max_prompt_length
            fb = getattr(self.env, "feedback_len", cfg.max_feedback_tokens)
            plan = self.memory_plan(target * len(mine), plen + cfg.num_turns * (max_new + fb) + 1)
            if not hasattr(self, "_opt_stash"):
                self._opt_stash, self._ref_stash = HostStash(), HostStash()
            if plan["grads"]:
                self._drop_grads()
            if plan["opt"]:
                self._opt_stash.park(plan["opt"])
        if batched:
            batch_tasks = [tasks[i % len(tasks)] for i in range(target)]
            for gi, trajs in enumerate(self.rollout_batch(batch_tasks, mine, max_new_tokens=max_new)):
                traj_groups.append((batch_tasks[gi], trajs))
                gen_tokens += sum(len(g) for t in trajs for g in t.gens)
                traj_tokens += sum(len(t.contexts[-1]) + len(t.gens[-1]) for t in trajs if t.gens)
                rewards_all.extend(M.kevin_trajectory_score([r.reward for r in t.results],
                                                            [r.correct for r in t.results]) for t in trajs)
                groups.append(self.samples_from_group(trajs, gi))
            kept = []
        elif cfg.dynamic_sampling and W == 1:
            kept, attempts = M.dynamic_sampling_refill(
                roll, target, min_std=cfg.starpo_min_std,
                max_attempts=cfg.max_sampling_attempts or 0,
                std_key=lambda g: M.group_reward_std([s.ret for s in g[0]]))
        elif cfg.dynamic_sampling:   # several ranks: refill decided on the gathered returns
            from .grpo_hooks import distributed_refill
            kept, attempts = distributed_refill(self.ctx, roll, target, min_std=cfg.starpo_min_std,
                                                max_attempts=cfg.max_sampling_attempts or 0)
        else:
            kept = [roll(i) for i in range(target)]
        for g, scores in kept:
            groups.append(g)
            rewards_all.extend(scores)
        ph.__exit__(None, None, None)
        if batched and self.rollout._num_pages is None:
            self.rollout.release_cache()          # the KV pool is rebuilt at the next rollout
        groups = self.assign_advantages(groups)
        samples = [s for g in groups for s in g]
        with pt.phase("ref_logp"):
            self.fill_ref_logps(samples, micro_batch_tokens)
        t_roll = time.time() - t0
        with pt.phase("offload"):
            if plan["ref"]:
                self._ref_stash.park(self._ref_slots())
            if plan["opt"]:
                self._opt_stash.restore(plan["opt"], self.ctx.device)
            if plan["grads"]:
                self._restore_grads()
        with pt.phase("update"):
            stats = self.update(samples, micro_batch_tokens)
        if getattr(self, "tp", None) is not None:
            with pt.phase("sync"):
                self.tp.shard.sync_from(self.w)      # in place: this rank's head / FFN slices
        if plan["ref"]:
            with pt.phase("offload"):
                self._ref_stash.restore(self._ref_slots(), self.ctx.device)
        self.step_idx += 1
        if self.curriculum is not None:
            self.curriculum.record([t for t, _ in traj_groups], [g for _, g in traj_groups])
        if self.search_hook is not None:
            rec = self.search_hook.maybe_run(self.step_idx, [t for t, _ in traj_groups],
                                             [g for _, g in traj_groups])
            if rec is not None:
                stats["search"] = rec
        stats.update({"step": self.step_idx, "reward_mean": sum(rewards_all) / max(1, len(rewards_all)),
                      "reward_std": M.group_reward_std(rewards_all), "groups": len(groups),
                      "samples": len(samples), "gen_tokens": gen_tokens, "traj_tokens": traj_tokens,
                      "adv_absmean": sum(abs(s.adv) for s in samples) / max(1, len(samples)),
                      "rollout_s": t_roll, "step_s": time.time() - t0,
                      "offload_opt_gb": round(sum(c[k].numel() * c[k].element_size() for c, k in plan["opt"]
                                                  if c[k] is not None) / 1e9, 2),
                      "dropped_grads": plan["grads"], "offload_ref": plan["ref"],
                      "grad_norm": self.trainer.opt.grad_norm()})
        stats.update({f"ms_{k}": v for k, v in pt.summary(self.ctx).items()})
        if self.ctx.is_main and (self.step_idx % max(1, cfg.logging_steps) == 0):
            log.event("grpo_step", **{k: (round(v, 5) if isinstance(v, float) else v) for k, v in stats.items()})
        return stats


def train_grpo(config: GRPOConfig, tasks: Optional[List[str]] = None, backend: str = "inprocess",
               env: Optional[RolloutEnv] = None, model_cfg=None, tokenizer=None) -> Dict[str, Any]:
    """Run ``config.total_steps`` GRPO steps (or until the plateau controller
    stops) and save an HF-format checkpoint to ``config.output_dir``."""
    from ..data.tokenizer import load_tokenizer
    from ..models.hf_io import load_pretrained_or_init, save_pretrained
    ctx = init_distributed()
    configure(config.output_dir)
    tok = tokenizer or load_tokenizer(config.model_id)
    weights = load_pretrained_or_init(config.model_id, ctx, model_cfg=model_cfg, bf16=config.bf16,
                                      seed=config.seed)
    if env is None:
        env = SyntheticRewardEnv(seed=config.seed, vocab_size=weights.cfg.vocab_size) \
            if config.reward_env == "synthetic" else _kernel_env(config)
    tr = GRPOTrainer(config, weights=weights, env=env, ctx=ctx, tokenizer=tok)
    tasks = list(tasks or ["synthetic-0"])
    history = []
    start = resume_grpo(tr, config.output_dir, ctx)
    for step in range(start, config.total_steps):
        k = config.tasks_per_step
        batch = [tasks[(step * k + i) % len(tasks)] for i in range(k)]
        st = tr.train_step(batch)
        history.append(st)
        if config.save_steps and (step + 1) % config.save_steps == 0:
            save_grpo_checkpoint(tr, weights, tok, config.output_dir, step + 1, ctx)
        if tr.controller is not None and tr.controller.update(step, st["reward_mean"]):
            log.info("adaptive stop", reason=tr.controller.stopped_reason)
            break
    if ctx.is_main:
        save_pretrained(weights, config.output_dir, tok)
    ctx.barrier()
    return {"output_dir": config.output_dir, "history": history}


def save_grpo_checkpoint(tr, weights, tok, output_dir: str, step: int, ctx) -> str:
    """``checkpoint-<step>``: HF weights + trainer_state (rank 0), and per rank
    the optimizer shard plus RNG states, so a GRPO run resumes mid-stage
    (the reference keeps weights only: kore/policy/grpo.py:906-928)."""
    import random as _random
    from ..models.hf_io import save_pretrained
    d = os.path.join(output_dir, f"checkpoint-{step}")
    if ctx.is_main:
        save_pretrained(weights, d, tok, keep_last=1, trainer_state={"global_step": step,
                                                                     "grpo_step_idx": tr.step_idx})
    ctx.barrier()
    state = {"opt": tr.trainer.opt.state_dict(), "py_rng": _random.getstate(),
             "torch_rng": torch.get_rng_state(), "step_idx": tr.step_idx,
             "cuda_rng": torch.cuda.get_rng_state() if torch.cuda.is_available() else None}
    torch.save(state, os.path.join(d, f"grpo_state-rank{ctx.rank}.pt"))
    ctx.barrier()
    return d


def resume_grpo(tr, output_dir: str, ctx) -> int:
    """Restore the latest checkpoint (weights, optimizer shard, RNG); returns the next step."""
    import random as _random
    from ..models.hf_io import load_weights
    from .configs import latest_checkpoint
    ck = latest_checkpoint(output_dir)
    if ck is None:
        return 0
    load_weights(tr.trainer.w, ck)
    step = json.load(open(os.path.join(ck, "trainer_state.json"))).get("global_step", 0)
    f = os.path.join(ck, f"grpo_state-rank{ctx.rank}.pt")
    if os.path.exists(f):
        st = torch.load(f, map_location="cpu", weights_only=False)
        tr.trainer.opt.load_state_dict(st["opt"])
        _random.setstate(st["py_rng"])
        torch.set_rng_state(st["torch_rng"])
        if st.get("cuda_rng") is not None and torch.cuda.is_available():
            torch.cuda.set_rng_state(st["cuda_rng"])
        tr.step_idx = st["step_idx"]
    if hasattr(tr, "sync_rollout_weights"):
        tr.sync_rollout_weights()
    log.info("grpo resumed", checkpoint=ck, step=step)
    return step


def _kernel_env(config: GRPOConfig):
    from ..env.kore_env import KernelRolloutEnv
    return KernelRolloutEnv(config)


def _main(argv: Optional[list] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print("usage: python -m kore_b200.policy.grpo <config.json>", file=sys.stderr)
        return 2
    raw = json.loads(Path(argv[0]).read_text())
    tasks = raw.get("tasks")
    cfg = grpo_config_from_dict(raw)
    out = train_grpo(cfg, tasks=tasks)
    print(f"[grpo] -> {out['output_dir']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
