"""Optional integrations of the GRPO loop.

Each piece is switched on by its ``GRPOConfig`` field and is inert otherwise:

* **curriculum** (``coevolve``): the step's tasks come from the open-ended
  :class:`CurriculumController` (learnability x regret x novelty frontier,
  deterministic for a seed and history, so every rank picks the same tasks)
  and every group's outcome is recorded back (success = any correct turn,
  regret = 1 - best speedup). Reference: kore/policy/grpo.py:2085-2098.
* **value prefilter** (``value_prefilter``): a turn samples
  ``num_candidates_per_turn`` responses sharing the prompt's KV pages, the
  value model ranks their kernels, only the top ``value_prefilter_k`` are
  verified, and the best verified one continues the trajectory.
  Reference: kore/policy/grpo.py:2415-2437.
* **search-then-distill** (``use_search``): every ``search_every`` steps rank
  0 runs the transform search from the step's best correct kernel and sends
  wins to the distillation sink. Reference: kore/policy/grpo.py:2225-2226.
* **agentic rollout** (``agentic``): trajectories are tool-using episodes of
  :class:`AgentHarness`; every assistant turn is one sample (its rendered
  conversation so far + its generation), turn rewards come from the turn's
  best tool evaluation, and the tool-use shaping is folded into the best
  correct turn. Reference: kore/policy/grpo.py:2503-2583.
* **distributed dynamic sampling**: with several ranks, degenerate groups
  (reward std <= min_std over ALL ranks' trajectories, gathered) are re-rolled
  up to the attempt budget; every rank sees the same gathered returns, so all
  keep the same groups. Reference: kore/policy/grpo.py:270-299 (DAPO refill).
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence

from ..env.base import TurnResult
from . import rl_math as M


# ----------------------------------------------------------------------------- curriculum
class CurriculumHook:
    """Co-evolution curriculum in the GRPO loop: the controller picks the
    step's tasks; per-task outcomes (solve rate, best verified speedup) are
    gathered over ranks before the archive update, so every rank serves the
    same tasks. Optional minting and competitor anchor from the config."""

    def __init__(self, trainer, space=None):
        from ..openended.controller import CoevolutionController
        from ..openended.proposer import Proposer
        cfg = trainer.cfg
        self.tr = trainer
        comp = None
        if getattr(cfg, "coevolve_regret_vs_opus", False) and getattr(cfg, "coevolve_opus_scores_path", None):
            from ..openended.competitor import build_competitor_scores, load_scores
            path = cfg.coevolve_opus_scores_path
            # a scores JSON, or the teacher's verified datagen records (JSONL) to mine them from
            comp = (build_competitor_scores([p for p in path.split(",") if p]) if path.endswith(".jsonl")
                    else load_scores(path)) or None
        self.ctrl = CoevolutionController(space=space, seed=cfg.seed, proposer=Proposer(competitor=comp),
                                          batch=cfg.coevolve_batch or 8, ctx=trainer.ctx,
                                          mint=bool(getattr(cfg, "coevolve_mint", False)),
                                          mint_batch=int(getattr(cfg, "coevolve_mint_batch", 6)))

    def choose(self, fallback: Sequence[Any], k: int) -> List[Any]:
        picked = self.ctrl.next_task_id(k)
        return picked if picked else list(fallback)[:k]

    def record(self, tasks: Sequence[Any], groups) -> None:
        out = []
        for task, trajs in zip(tasks, groups):
            res = [r for t in trajs for r in t.results]
            rate = sum(1 for r in res if r.correct) / max(1, len(res))
            speed = max((getattr(r.obs, "speedup", None) or 0.0 for r in res
                         if r.correct and r.obs is not None), default=0.0)
            out.append((str(task), rate, speed if rate > 0 else None))
        self.ctrl.record_batch(out)


# ----------------------------------------------------------------------------- value prefilter
class ValuePrefilter:
    def __init__(self, trainer):
        from ..value.model import ValueModel
        cfg = trainer.cfg
        self.k = max(1, int(cfg.value_prefilter_k))
        self.n = max(self.k, int(cfg.num_candidates_per_turn))
        self.model = None
        if cfg.value_model_path:
            with open(cfg.value_model_path) as f:
                self.model = ValueModel.from_json(f.read())

    def pick(self, codes: Sequence[str], task=None) -> List[int]:
        """Indices of the candidates to verify: the value model's top k, or the
        schedule heuristic's when no (or only a degenerate) model is loaded."""
        if len(codes) <= self.k:
            return list(range(len(codes)))
        from ..value.rerank import rank_candidates
        return rank_candidates(list(codes), task=task, model=self.model)[: self.k]


# ----------------------------------------------------------------------------- search -> distill
class SearchDistill:
    def __init__(self, trainer):
        from .distill import DistillSink
        cfg = trainer.cfg
        self.tr = trainer
        self.every = max(1, int(cfg.search_every))
        self.sink = DistillSink(cfg.coevolve_distill_path, min_speedup=cfg.coevolve_distill_min_speedup)
        self.runs: List[Dict] = []

    def maybe_run(self, step: int, tasks: Sequence[Any], groups) -> Optional[Dict]:
        tr, cfg = self.tr, self.tr.cfg
        if not tr.ctx.is_main or step % self.every != 0:
            return None
        best = None
        for task, trajs in zip(tasks, groups):
            for t in trajs:
                for r in t.results:
                    if r.correct and r.code and (best is None or r.reward > best[0]):
                        best = (r.reward, task, r.code)
        if best is None or not hasattr(tr.env, "_env"):
            return None
        from ..search.propose import search_from_kernel
        _, task, code = best
        kenv = tr.env._env(task)
        res = search_from_kernel(code, kenv, budget=cfg.search_budget, k_expand=cfg.search_k_expand,
                                 max_depth=cfg.search_max_depth or 6, bnb=cfg.search_bnb,
                                 task=getattr(kenv, "task", None),
                                 value_fn="model" if getattr(cfg, "search_value_prior", True) else None)
        won = False
        if res.best_src and res.best_score:
            won = self.sink.add(str(task), res.best_src, float(res.best_score),
                                operation=getattr(kenv.task, "operation", None))
            if won:
                self.sink.flush()
        rec = {"step": step, "task": str(task), "best_speedup": res.best_score, "evaluated": res.evaluated,
               "distilled": won}
        self.runs.append(rec)
        return rec


# ----------------------------------------------------------------------------- agentic
class EngineChatPolicy:
    """The policy an :class:`AgentHarness` talks to: renders the conversation
    with the tokenizer, samples one response on the rollout engine, and records
    (prompt ids, generated ids, log-probs, finish reason) per assistant turn."""

    def __init__(self, trainer, max_new: int, seed: int):
        self.tr = trainer
        self.max_new = max_new
        self.seed = seed
        self.turns: List[tuple] = []

    def generate(self, messages: List[dict]) -> str:
        from ..data.tokenizer import render_chat
        from ..engine.rollout import GenRequest
        tr, cfg = self.tr, self.tr.cfg
        ids, _ = render_chat(tr.tok, messages, add_generation_prompt=True)
        ids = list(ids)[-cfg.max_prompt_length:]
        out = tr.rollout.generate([GenRequest(ids, self.max_new, rid=0)], temperature=cfg.temperature,
                                  top_p=cfg.top_p, eos_ids=tr.eos, seed=self.seed + 131 * len(self.turns))[0]
        self.turns.append((ids, list(out.tokens), list(out.logps), out.finish_reason))
        return tr.tok.decode(out.tokens, skip_special_tokens=True)


def rollout_agentic(trainer, task, traj_ids: Sequence[int], max_new: int):
    """One tool-using episode per trajectory; returns ``Trajectory`` objects
    whose turns are the episode's assistant turns."""
    from ..agent.harness import AgentHarness
    from .grpo import Trajectory
    cfg = trainer.cfg
    kenv = trainer.env._env(task)
    out = []
    for t in traj_ids:
        pol = EngineChatPolicy(trainer, max_new, seed=cfg.seed * 7919 + trainer.step_idx * 97 + t)
        ep = AgentHarness(kenv, kenv.task, max_turns=cfg.max_tool_turns,
                          transforms=cfg.agentic_transform_tools).run(pol)
        rewards = list(ep.turn_rewards)
        correct = list(ep.turn_correct)
        if any(correct):   # tool-use shaping, once, on the best correct turn
            bi = max((i for i, c in enumerate(correct) if c), key=lambda i: rewards[i])
            rewards[bi] += cfg.tool_reward_weight * ep.tool_reward
        n = min(len(pol.turns), len(rewards))
        tr = Trajectory(t)
        for i in range(n):
            ids, gen, lps, fin = pol.turns[i]
            tr.contexts.append(ids)
            tr.gens.append(gen)
            tr.gen_logps.append(lps)
            tr.finish.append(fin)
            tr.results.append(TurnResult(reward=float(rewards[i]), correct=bool(correct[i]),
                                         code=ep.codes[i] if i < len(ep.codes) else "",
                                         phi=ep.turn_phis[i] if i < len(ep.turn_phis) else None))
        out.append(tr)
    return out


# ----------------------------------------------------------------------------- distributed refill
def distributed_refill(ctx, roll, target: int, *, min_std: float, max_attempts: int = 0):
    """DAPO dynamic sampling over ranks: ``roll(attempt) -> (samples, scores)``
    is called on every rank with the same attempt index; a group is kept when
    the std of its returns gathered from all ranks exceeds ``min_std``."""
    max_attempts = max_attempts or 3 * target
    kept, attempts = [], 0
    while len(kept) < target and attempts < max_attempts:
        g = roll(attempts)
        attempts += 1
        full = M.merge_across_ranks(ctx.all_gather_object([s.ret for s in g[0]]))
        if M.group_reward_std(full) > min_std:
            kept.append(g)
    return kept, attempts
