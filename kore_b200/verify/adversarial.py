"""Adversarial input battery and coevolved test genomes.

``battery(inputs)`` yields deterministic hard regimes (zeros, huge/tiny
magnitudes, denormals, near ties, alternating signs, sparse spikes, one-hot
rows). ``coevolve_tests`` evolves input "genomes" (regime + scale + sparsity
+ seed) that maximise the disagreement between a candidate and the oracle,
so a candidate that is only correct on benign inputs is caught. Reference
parity: kore/verify/adversarial.py:66-168 and :535-1062.
"""
from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Callable, Iterator, List, Sequence, Tuple

import torch

REGIMES = ("zeros", "large", "tiny", "denormal", "near_tie", "alternating", "sparse_spike", "one_hot")


def apply_regime(t: torch.Tensor, regime: str, scale: float = 1.0, sparsity: float = 0.001,
                 seed: int = 0) -> torch.Tensor:
    if not t.is_floating_point():
        return t
    g = torch.Generator(device=t.device)
    g.manual_seed(seed)
    x = t.clone()
    if regime == "zeros":
        x.zero_()
    elif regime == "large":
        x.mul_(100.0 * scale)
    elif regime == "tiny":
        x.mul_(1e-3 / max(scale, 1e-6))
    elif regime == "denormal":
        x.copy_(torch.full_like(x.float(), 1e-39).to(x.dtype))
    elif regime == "near_tie":
        x.copy_((1.0 + 1e-3 * x.float()).to(x.dtype))
    elif regime == "alternating":
        sign = torch.ones(x.numel(), device=x.device)
        sign[1::2] = -1
        x.copy_((x.float().abs() * sign.view(x.shape) * scale).to(x.dtype))
    elif regime == "sparse_spike":
        m = torch.rand(x.shape, generator=g, device=x.device) < sparsity
        x.masked_fill_(m, 50.0 * scale)
    elif regime == "one_hot" and x.dim() >= 2:
        x.zero_()
        idx = torch.randint(0, x.shape[-1], x.shape[:-1], generator=g, device=x.device)
        x.scatter_(-1, idx.unsqueeze(-1), scale)
    return x


def battery(inputs: Sequence[torch.Tensor]) -> Iterator[Tuple[str, Tuple[torch.Tensor, ...]]]:
    for r in REGIMES:
        yield r, tuple(apply_regime(t, r) for t in inputs)


@dataclass
class Genome:
    regime: str
    scale: float
    sparsity: float
    seed: int

    def mutate(self, rng: random.Random) -> "Genome":
        return Genome(rng.choice(REGIMES) if rng.random() < 0.3 else self.regime,
                      max(1e-3, self.scale * rng.choice((0.5, 2.0, 1.0))),
                      min(0.5, max(1e-5, self.sparsity * rng.choice((0.1, 10.0, 1.0)))), rng.randrange(1 << 30))


def coevolve_tests(make_inputs: Callable[[int], Sequence[torch.Tensor]], candidate: Callable, oracle: Callable,
                   score: Callable[[torch.Tensor, torch.Tensor], float], *, population: int = 8,
                   generations: int = 4, seed: int = 0) -> List[Tuple[Genome, float]]:
    """Evolve genomes maximising ``score(candidate_out, oracle_out)`` (an error,
    higher = worse candidate). Returns the final population sorted worst-first."""
    rng = random.Random(seed)
    pop = [Genome(rng.choice(REGIMES), 1.0, 1e-3, rng.randrange(1 << 30)) for _ in range(population)]

    def fitness(gn: Genome) -> float:
        ins = tuple(apply_regime(t, gn.regime, gn.scale, gn.sparsity, gn.seed) for t in make_inputs(gn.seed))
        try:
            return float(score(candidate(*ins), oracle(*ins)))
        except Exception:  # noqa: BLE001 - a crash on this input is maximal disagreement
            return float("inf")

    scored = [(g, fitness(g)) for g in pop]
    for _ in range(generations):
        scored.sort(key=lambda p: p[1], reverse=True)
        elite = scored[: max(1, population // 2)]
        kids = [(c, fitness(c)) for c in (rng.choice(elite)[0].mutate(rng) for _ in range(population - len(elite)))]
        scored = elite + kids
    scored.sort(key=lambda p: p[1], reverse=True)
    return scored
