"""AlphaKernel on scripted graders: transposition DAG, MAX backup, LCB
discipline, successive halving, budget, branch-and-bound, repairable
incorrect nodes and the propose fail-safe."""
import math
import random
import re

from kore_b200.search import (AlphaKernel, Budget, Eval, MeasureStats, RooflineCeiling, TransformProposePolicy,
                              fingerprint, search, successive_halving)
from kore_b200.search.bandit import rung_schedule
from kore_b200.transform.budget import ErrorBudget

SRC = """import triton
import triton.language as tl


@triton.jit
def k(X, Y, N, BLOCK: tl.constexpr):
    x = tl.exp(tl.load(X))


def run(x):
    k[(1,)](x, x, 1, BLOCK=128, num_warps=4)
"""


def _block(src):
    return int(re.search(r"BLOCK=(\d+)", src).group(1))


def test_fingerprint_ignores_cosmetics():
    assert fingerprint(SRC) == fingerprint(SRC.replace("    x =", "    x  =") + "\n# note\n")
    assert fingerprint(SRC) != fingerprint(SRC.replace("BLOCK=128", "BLOCK=256"))


def test_measure_stats_lcb_and_rungs():
    s = MeasureStats()
    assert s.lcb() == -math.inf
    s.add(2.0)
    assert s.lcb() < 2.0
    for x in (2.0, 2.0, 2.0):
        s.add(x)
    assert abs(s.lcb() - 2.0) < 1e-12
    r = rung_schedule(8, 64, eta=2)
    assert r[0] == 1 and sum(p * max(1, 8 // 2 ** i) for i, p in enumerate(r)) <= 64


def test_lcb_prefers_stable_over_noisy():
    rng = random.Random(1)
    arms = {"noisy": lambda: 1.6 + rng.choice([-1.2, 1.2]), "stable": lambda: 1.5 + rng.gauss(0, 0.01)}
    best = successive_halving(list(arms), lambda a: arms[a](), Budget(40), eta=1)
    assert best == "stable"


def test_budget_respected_and_search_improves():
    calls = []

    def ev(src):
        calls.append(src)
        return 1.0 + math.log2(_block(src)) / 10
    r = search(SRC, ev, budget=10, eps_budget=ErrorBudget(total=1.0))
    assert len(calls) == r.evaluated <= 10
    assert r.best_score > 1.0 + math.log2(128) / 10 and r.path


def test_transposition_links_instead_of_regrading():
    graded = []

    def ev(src):
        graded.append(fingerprint(src))
        return 1.0
    ak = AlphaKernel(ev, budget=60, k_expand=16, max_depth=3, eps_budget=ErrorBudget(total=1.0), sh_max_measures=1)
    ak.run(SRC)
    assert ak.counters["linked"] > 0                      # e.g. warps 4->8->4 style cycles and commuting edits
    assert len(set(graded)) == len(graded)                # no kernel graded twice (no re-measure at sh_max=1)


def test_max_backup_and_repairable_incorrect():
    def ev(src):
        if "num_warps=8" in src and "BLOCK=256" not in src:
            return None                                   # incorrect, but a later edit repairs it
        if "num_warps=8" in src and "BLOCK=256" in src:
            return 3.0
        return 1.0
    ak = AlphaKernel(ev, budget=80, k_expand=20, max_depth=3, eps_budget=ErrorBudget(total=1.0), sh_max_measures=1)
    r = ak.run(SRC)
    assert r.best_score == 3.0
    root = ak.nodes[0]
    assert root.best >= 3.0 - 0.3                         # the best descendant's LCB reaches the root


def test_branch_and_bound_prunes_dominated_nodes():
    def ev(src):
        return 2.0
    ceil = RooflineCeiling(t_min_ms=1.0, baseline_ms=1.5, safety_margin=0.0)   # nothing can beat 1.5x
    ak = AlphaKernel(ev, budget=30, k_expand=4, ceiling_fn=ceil, bnb=True, eps_budget=ErrorBudget(total=1.0))
    r = ak.run(SRC)
    assert ak.counters["pruned"] > 0 and r.evaluated < 30


def test_propose_fail_safe_on_torch_source():
    pol = TransformProposePolicy()
    assert pol.propose("import torch\n\ndef f(x):\n    return x * 2\n") == []
    assert pol.propose(SRC) and TransformProposePolicy(discover=True).propose(SRC)


def test_model_value_prior_is_memoised_and_orders_sources():
    from kore_b200.search.propose import model_value_fn
    f = model_value_fn()
    good = "acc = tl.zeros((BLOCK_M, BLOCK_N), dtype=tl.float32)\nBLOCK_M = 128\nacc += tl.dot(a, b)\n"
    bad = "BLOCK_M = 8\nacc += tl.sum(a * b)\n"
    assert f(good) > f(bad) and f(good) == f(good)
