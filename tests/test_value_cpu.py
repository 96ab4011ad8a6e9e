"""Value-model reranking: heuristic cold start, degenerate-model fallback,
trained-model ordering, replay-validation metrics."""
import math

import numpy as np

from kore_b200.value.model import ValueModel, features
from kore_b200.value.rerank import (benches_to_best, expected_random_benches, heuristic_score, rank_candidates,
                                    score_candidates, spearman)

GOOD = """@triton.jit
def k(A, B, C, BM: tl.constexpr):
    acc = tl.zeros((BM, BM), dtype=tl.float32)
    for k in range(0, K, BK):
        a = tl.load(A, mask=m)
        acc += tl.dot(a, b)
run: k[(1,)](BM=128, BN=128, BK=64, num_warps=8, num_stages=3)
"""
BAD = "def k(x):\n    return x  # BLOCK=8 num_warps=32\n"


def test_heuristic_cold_start():
    assert heuristic_score(GOOD) > heuristic_score(BAD)
    assert rank_candidates([BAD, GOOD]) == [1, 0]
    s = score_candidates([GOOD, GOOD + " "])
    assert s[0] != s[1]                                   # tie-breaker separates distinct sources


def test_degenerate_model_defers_to_heuristic():
    m = ValueModel()
    F = np.stack([features(GOOD), features(BAD)])
    m.fit(F, np.array([1, 1]), np.array([1, 1]), np.array([0.0, 0.0]))
    m.w_speed[:] = 0.0
    m.w_compile[:] = 0.0
    m.w_snr[:] = 0.0
    assert rank_candidates([BAD, GOOD], model=m) == [1, 0]


def test_trained_model_orders_by_measured_speed():
    srcs = [GOOD.replace("BM=128", f"BM={b}") for b in (16, 32, 64, 128, 256)]
    F = np.stack([features(s) for s in srcs])
    ls = np.array([math.log2(b) / 10 for b in (16, 32, 64, 128, 256)])
    m = ValueModel().fit(F, np.ones(5), np.ones(5), ls)
    order = rank_candidates(srcs, model=m)
    assert order[0] == 4
    pred = score_candidates(srcs, model=m)
    assert spearman(pred, list(ls)) > 0.9


def test_replay_metrics():
    assert benches_to_best([2, 0, 1], [1.0, None, 3.0]) == 1
    assert benches_to_best([0, 1], [None, None]) is None
    assert expected_random_benches(7) == 4.0
    assert abs(spearman([1, 2, 3], [3, 2, 1]) + 1) < 1e-12
