"""Structured adversarial inputs and the co-evolution that grows them.

A random-input check admits lucky passes: a kernel wrong only on a thin
slice of the input domain (exact zeros, denormals, values near overflow, all
equal rows, activation kinks, isolated spikes) sails through ``randn``
trials. :func:`battery` replays a fixed list of such regimes, per operand slot
(only that operand perturbed) and for all operands at once, with
magnitudes chosen for the storage dtype so a correct kernel is stressed
without being forced to overflow.

:func:`coevolve_tests` evolves parametric test genomes (regime, scale,
sparsity, kink offset, seed) to maximise a candidate's error against the
oracle under a minimal criterion: a genome is kept only if the oracle is
finite on it (a test the reference itself cannot answer is not a test) and
it is novel against the archive of already-found breaks.
:func:`random_search` is the undirected control at equal budget, and
:func:`fold_breaking_cases` turns discovered breaks into extra deterministic
cases for the equivalence oracle.

Reference behaviour: kore/verify/adversarial.py:66-1062 (patterns,
dtype-aware magnitudes, per-slot emission, minimal-criterion co-evolution,
random-search control, folding).
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass
from typing import Callable, Iterator, List, Optional, Sequence, Tuple

import torch

# magnitude that a correct kernel survives in each storage dtype (about a
# hundredth of the dtype's max, so x^2 or exp-like ops still overflow only
# where the reference does)
_BIG = {torch.float16: 300.0, torch.bfloat16: 1e4, torch.float32: 1e6, torch.float64: 1e9}
_TINY = {torch.float16: 1e-7, torch.bfloat16: 1e-38, torch.float32: 1e-39, torch.float64: 1e-310}
KNOTS = (0.0, 1.0, -1.0, 3.0, -3.0, 6.0, -6.0, 0.5, -0.5, 2.0)

PATTERNS = ("zeros", "ones", "neg_ones", "all_equal", "large_pos", "large_neg", "small_pos", "denormal",
            "signed_ramp", "sign_alternating", "sparse_spikes", "inf_adjacent_pos", "inf_adjacent_neg",
            "activation_knots", "mixed_magnitude", "near_tie", "one_hot")
_PRIOR = ("large_pos", "activation_knots", "large_neg", "denormal", "sparse_spikes", "inf_adjacent_pos",
          "mixed_magnitude", "zeros")
# names of the earlier battery, still accepted by apply_regime
REGIMES = ("zeros", "large", "tiny", "denormal", "near_tie", "alternating", "sparse_spike", "one_hot")
_ALIAS = {"large": "large_pos", "tiny": "small_pos", "alternating": "sign_alternating",
          "sparse_spike": "sparse_spikes"}


def _dt(t: torch.Tensor) -> torch.dtype:
    return t.dtype if t.dtype in _BIG else torch.float32


def apply_regime(t: torch.Tensor, regime: str, scale: float = 1.0, sparsity: float = 0.001,
                 seed: int = 0, offset: float = 0.0) -> torch.Tensor:
    """``t`` (same shape, dtype, device) rewritten into an input regime."""
    if not t.is_floating_point():
        return t
    regime = _ALIAS.get(regime, regime)
    g = torch.Generator(device="cpu").manual_seed(int(seed) & 0x7FFFFFFF)
    dt = _dt(t)
    big, tiny = _BIG[dt], _TINY[dt]
    n = t.numel()
    base = t.detach().float().cpu().reshape(-1)
    if regime == "zeros":
        x = torch.zeros(n)
    elif regime == "ones":
        x = torch.ones(n) * scale
    elif regime == "neg_ones":
        x = -torch.ones(n) * scale
    elif regime == "all_equal":
        x = torch.full((n,), float(1.7 * scale))
    elif regime == "large_pos":
        x = base.abs() * min(big, 100.0 * scale)
    elif regime == "large_neg":
        x = -base.abs() * min(big, 100.0 * scale)
    elif regime == "small_pos":
        x = base.abs() * 1e-3 / max(scale, 1e-6)
    elif regime == "denormal":
        x = torch.full((n,), tiny * 10) * torch.sign(base + 1e-30)
    elif regime == "signed_ramp":
        x = torch.linspace(-4.0 * scale, 4.0 * scale, n)
    elif regime == "sign_alternating":
        s = torch.ones(n)
        s[1::2] = -1
        x = base.abs() * s * scale
    elif regime == "sparse_spikes":
        x = base.clone()
        m = torch.rand(n, generator=g) < sparsity
        x[m] = 50.0 * scale * torch.sign(torch.randn(int(m.sum()), generator=g))
    elif regime == "inf_adjacent_pos":
        x = torch.full((n,), big) * (1.0 + 0.01 * base.abs().clamp(max=1.0))
    elif regime == "inf_adjacent_neg":
        x = -torch.full((n,), big) * (1.0 + 0.01 * base.abs().clamp(max=1.0))
    elif regime == "activation_knots":
        k = torch.tensor(KNOTS)
        x = k[torch.randint(0, len(KNOTS), (n,), generator=g)] + offset
    elif regime == "mixed_magnitude":
        e = torch.randint(-20, 21, (n,), generator=g).float()
        x = torch.sign(base + 1e-30) * torch.pow(2.0, e).clamp(max=big)
    elif regime == "near_tie":
        x = 1.0 + 1e-3 * base
    elif regime == "one_hot" and t.dim() >= 2:
        x = torch.zeros(t.shape)
        idx = torch.randint(0, t.shape[-1], t.shape[:-1], generator=g)
        x.scatter_(-1, idx.unsqueeze(-1), float(scale))
        x = x.reshape(-1)
    else:
        x = base
    return x.reshape(t.shape).to(device=t.device, dtype=t.dtype)


def battery(inputs: Sequence[torch.Tensor], dtype: Optional[str] = None
            ) -> Iterator[Tuple[str, Tuple[torch.Tensor, ...]]]:
    """Every pattern applied to all floating operands at once, then, for
    multi-operand inputs, to one operand slot at a time."""
    ins = tuple(inputs)
    floats = [i for i, t in enumerate(ins) if torch.is_tensor(t) and t.is_floating_point()]
    for p in PATTERNS:
        yield p, tuple(apply_regime(t, p, seed=i) if i in floats else t for i, t in enumerate(ins))
    if len(floats) > 1:
        for slot in floats:
            for p in PATTERNS:
                yield f"{p}@{slot}", tuple(apply_regime(t, p, seed=i) if i == slot else t for i, t in enumerate(ins))


@dataclass
class Genome:
    regime: str
    scale: float
    sparsity: float
    seed: int
    offset: float = 0.0
    slot: int = -1                  # -1: every operand

    def mutate(self, rng: random.Random) -> "Genome":
        return Genome(rng.choice(PATTERNS) if rng.random() < 0.3 else self.regime,
                      max(1e-3, self.scale * rng.choice((0.5, 2.0, 1.0, 10.0, 0.1))),
                      min(0.5, max(1e-5, self.sparsity * rng.choice((0.1, 10.0, 1.0)))),
                      rng.randrange(1 << 30),
                      self.offset + rng.choice((0.0, 1e-3, -1e-3, 1e-6, -1e-6)),
                      self.slot if rng.random() < 0.8 else rng.choice((-1, 0, 1)))

    def crossover(self, other: "Genome", rng: random.Random) -> "Genome":
        """Uniform crossover: each field from one parent or the other."""
        pick = lambda a, b: a if rng.random() < 0.5 else b          # noqa: E731
        return Genome(pick(self.regime, other.regime), pick(self.scale, other.scale),
                      pick(self.sparsity, other.sparsity), rng.randrange(1 << 30),
                      pick(self.offset, other.offset), pick(self.slot, other.slot))

    def key(self) -> Tuple:
        return (self.regime, round(math.log10(self.scale), 1), self.slot)

    def inputs(self, base: Sequence[torch.Tensor]) -> Tuple[torch.Tensor, ...]:
        return tuple(apply_regime(t, self.regime, self.scale, self.sparsity, self.seed + i, self.offset)
                     if (self.slot < 0 or self.slot == i) else t for i, t in enumerate(base))


def _fitness(g: Genome, make_inputs, candidate, oracle, score) -> float:
    """Error of the candidate (the worst of several, when a list is given) on
    the genome's inputs; -inf when the oracle itself has no finite answer."""
    ins = g.inputs(tuple(make_inputs(g.seed)))
    try:
        ref = oracle(*ins)
    except Exception:  # noqa: BLE001 - undefined for the reference: not a valid test
        return -math.inf
    if not bool(torch.isfinite(ref.float()).all()):
        return -math.inf                     # minimal criterion: the oracle must answer
    worst = -math.inf
    for c in (candidate if isinstance(candidate, (list, tuple)) else [candidate]):
        try:
            worst = max(worst, float(score(c(*ins), ref)))
        except Exception:  # noqa: BLE001 - a crash on a valid input is maximal disagreement
            return math.inf
    return worst


def coevolve_tests(make_inputs: Callable[[int], Sequence[torch.Tensor]], candidate: Callable, oracle: Callable,
                   score: Callable[[torch.Tensor, torch.Tensor], float], *, population: int = 8,
                   generations: int = 4, seed: int = 0, novelty_bonus: float = 0.0,
                   crossover_rate: float = 0.5, archive: Optional[dict] = None) -> List[Tuple[Genome, float]]:
    """Evolve genomes maximising ``score(candidate_out, oracle_out)`` (an
    error: higher means a worse candidate; ``candidate`` may be a list, scored
    by its worst member). Children come from crossover of two elites (with
    probability ``crossover_rate``) followed by mutation. ``archive``, when
    given, keeps the highest error seen per genome niche (pattern, scale
    decade, operand). Returns the final population, worst candidate error
    first; genomes invalid for the oracle score -inf."""
    rng = random.Random(seed)
    # stratified start: distinct patterns, the historically most breaking first
    order = list(_PRIOR) + [p for p in PATTERNS if p not in _PRIOR]
    pop = [Genome(order[(seed + i) % len(order)], 1.0, 1e-3, rng.randrange(1 << 30)) for i in range(population)]
    seen: dict = {}

    def fit(g: Genome) -> float:
        f = _fitness(g, make_inputs, candidate, oracle, score)
        if archive is not None and f > archive.get(g.key(), (-math.inf, None))[0]:
            archive[g.key()] = (f, g)
        if novelty_bonus and math.isfinite(f):
            f += novelty_bonus / (1 + seen.get(g.key(), 0))
        seen[g.key()] = seen.get(g.key(), 0) + 1
        return f

    scored = [(g, fit(g)) for g in pop]
    for _ in range(generations):
        scored.sort(key=lambda p: p[1], reverse=True)
        elite = [p for p in scored[: max(1, population // 2)] if p[1] > -math.inf] or scored[:1]
        kids = []
        for _ in range(population - len(elite)):
            a = rng.choice(elite)[0]
            if len(elite) > 1 and rng.random() < crossover_rate:
                a = a.crossover(rng.choice(elite)[0], rng)
            kids.append(a.mutate(rng))
        scored = elite + [(c, fit(c)) for c in kids]
    scored.sort(key=lambda p: p[1], reverse=True)
    return scored


def random_search(make_inputs, candidate, oracle, score, *, budget: int = 32, seed: int = 0
                  ) -> List[Tuple[Genome, float]]:
    """Undirected control: ``budget`` independent random genomes."""
    rng = random.Random(seed)
    out = []
    for _ in range(budget):
        g = Genome(rng.choice(PATTERNS), 10 ** rng.uniform(-3, 3), 10 ** rng.uniform(-5, -0.5),
                   rng.randrange(1 << 30), rng.choice((0.0, 1e-3, -1e-3)), rng.choice((-1, 0, 1)))
        out.append((g, _fitness(g, make_inputs, candidate, oracle, score)))
    out.sort(key=lambda p: p[1], reverse=True)
    return out


def fold_breaking_cases(genomes: Sequence[Tuple[Genome, float]], threshold: float
                        ) -> Callable[[Sequence[torch.Tensor]], List[Tuple[str, Tuple[torch.Tensor, ...]]]]:
    """An ``adversarial_inputs_fn`` for the equivalence oracle that replays
    every genome whose error exceeded ``threshold``."""
    keep = [g for g, e in genomes if e > threshold and e > -math.inf]

    def extra(base: Sequence[torch.Tensor]):
        return [(f"folded:{g.regime}:{g.seed}", g.inputs(tuple(base))) for g in keep]
    return extra
