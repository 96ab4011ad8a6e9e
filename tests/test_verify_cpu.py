"""Equivalence oracle prongs, pure verdict, strict non-finite comparison,
per-slot adversarial battery, metamorphic relations, determinism, and
folding co-evolved breaks back into the battery."""
import math

import torch

from kore_b200.verify.adversarial import (PATTERNS, battery, coevolve_tests, fold_breaking_cases,
                                          random_search)
from kore_b200.verify.equivalence import (ProngResult, Tolerance, compare, equivalence_verdict,
                                          false_accept_probability, tolerance_for, verify_equivalence)
from kore_b200.verify import metamorphic as mm


def mk1(s):
    return (torch.randn(32, 64, generator=torch.Generator().manual_seed(s)),)


def mk2(s):
    g = torch.Generator().manual_seed(s)
    return torch.randn(32, 64, generator=g), torch.randn(32, 64, generator=g)


def test_pure_verdict_and_bound():
    tol = Tolerance()
    v = equivalence_verdict([ProngResult("random", True, comparisons=10 ** 6), ProngResult("adversarial", True)], tol)
    assert v.verified and v.confidence > 0.99 and v.first_failure is None
    v = equivalence_verdict([ProngResult("random", True, comparisons=100), ProngResult("metamorphic", False),
                             ProngResult("determinism", False)], tol)
    assert not v.verified and v.first_failure == "metamorphic"
    assert abs(false_accept_probability(0.01, 100) - 0.99 ** 100) < 1e-12
    assert tolerance_for("bf16").rtol > tolerance_for("fp32").rtol and tolerance_for("fp8_e4m3").snr_db_min < 20


def test_non_finite_positions_are_strict():
    r = torch.tensor([1.0, float("inf"), float("nan"), -float("inf")])
    assert compare(r.clone(), r, 1e-3, 1e-6, 40).ok
    assert not compare(torch.tensor([1.0, float("inf"), 0.0, -float("inf")]), r, 1e-3, 1e-6, 40).ok
    assert not compare(torch.tensor([1.0, -float("inf"), float("nan"), -float("inf")]), r, 1e-3, 1e-6, 40).ok


def test_battery_covers_patterns_per_slot():
    cases = list(battery(mk2(0)))
    assert len(cases) == 3 * len(PATTERNS)
    labels = [c[0] for c in cases]
    assert "denormal@1" in labels and "activation_knots" in labels
    # a binary kernel that is wrong only when its SECOND operand is large
    ref = lambda a, b: a * torch.tanh(b)
    cand = lambda a, b: torch.where(b.abs() > 20, a, a * torch.tanh(b))
    v = verify_equivalence(cand, ref, mk2, "fp32", op_class="binary")
    assert v.prongs["random"].passed and not v.prongs["adversarial"].passed


def test_metamorphic_catches_a_hidden_reduction():
    ref = lambda x: torch.relu(x)
    sneaky = lambda x: torch.relu(x) + 0.05 * x.mean()           # depends on other elements
    v = verify_equivalence(sneaky, ref, mk1, "fp32", op_class="elementwise", adversarial=False,
                           tol=Tolerance(rtol=1e-2, atol=1e-2, snr_db_min=20, metamorphic_rtol=1e-5))
    assert v.prongs["random"].passed and not v.prongs["metamorphic"].passed
    assert mm.relations_for("softmax") and mm.relations_for("gemm") == []
    ok, _ = mm.reduction_inrow_permutation(lambda x: x.sum(-1), mk1(0)[0])
    assert ok


def test_determinism_prong():
    noisy = lambda x: x + 1e-3 * torch.randn_like(x)
    v = verify_equivalence(noisy, lambda x: x, mk1, "fp32", adversarial=False, metamorphic=False,
                           tol=Tolerance(rtol=1e-2, atol=1e-2, snr_db_min=20))
    assert v.prongs["random"].passed and not v.prongs["determinism"].passed and not v.verified


def test_good_kernel_verifies_with_confidence():
    v = verify_equivalence(lambda x: torch.softmax(x, -1), lambda x: torch.softmax(x.double(), -1).float(), mk1,
                           "fp32", op_class="softmax")
    assert v.verified and v.confidence > 0.5, v.details


def test_coevolved_breaks_fold_into_the_oracle():
    ref = lambda x: torch.softmax(x.double(), -1).float()
    naive = lambda x: torch.exp(x) / torch.exp(x).sum(-1, keepdim=True)
    err = lambda a, b: float((a.float() - b.float()).abs().max()) if torch.isfinite(a).all() else math.inf
    pop = coevolve_tests(mk1, naive, ref, err, population=8, generations=3)
    assert pop[0][1] > 1e-3
    extra = fold_breaking_cases(pop, 1e-3)
    v = verify_equivalence(naive, ref, mk1, "fp32", adversarial=False, metamorphic=False, determinism=False)
    assert v.verified                                        # random inputs alone miss it
    v = verify_equivalence(naive, ref, mk1, "fp32", metamorphic=False, determinism=False,
                           adversarial_inputs_fn=extra)
    assert not v.verified and v.first_failure == "adversarial"
    ctrl = random_search(mk1, naive, ref, err, budget=8)
    assert len(ctrl) == 8


def test_coevolution_crossover_archive_and_candidate_sets():
    import math
    import random

    import torch

    from kore_b200.verify.adversarial import Genome, coevolve_tests

    def make(seed):
        return (torch.randn(64, 16, generator=torch.Generator().manual_seed(seed)),)
    oracle = lambda x: torch.softmax(x.float(), -1)                      # noqa: E731
    good = oracle
    naive = lambda x: torch.exp(x.float()) / torch.exp(x.float()).sum(-1, keepdim=True)   # overflows at large x
    score = lambda o, r: float((o.float() - r).abs().nan_to_num(1e9).max())                # noqa: E731
    arch = {}
    pop = coevolve_tests(make, [good, naive], oracle, score, population=8, generations=4, seed=1, archive=arch)
    assert pop[0][1] > 1e-3 and arch and max(v[0] for v in arch.values()) == pop[0][1]
    only_good = coevolve_tests(make, good, oracle, score, population=6, generations=2, seed=1)
    assert only_good[0][1] < 1e-5
    a, b = Genome("zeros", 1.0, 1e-3, 1), Genome("huge", 100.0, 1e-2, 2, 1e-3, 0)
    c = a.crossover(b, random.Random(0))
    assert c.regime in ("zeros", "huge") and c.scale in (1.0, 100.0) and c.slot in (-1, 0)
