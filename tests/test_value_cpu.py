"""Value-model reranking: heuristic cold start, degenerate-model fallback,
trained-model ordering, replay-validation metrics."""
import math

import numpy as np
import pytest

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
    m = ValueModel("v1")
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
    m = ValueModel("v1").fit(F, np.ones(5), np.ones(5), ls)
    order = rank_candidates(srcs, model=m)
    assert order[0] == 4
    pred = score_candidates(srcs, model=m)
    assert spearman(pred, list(ls)) > 0.9


def test_replay_metrics():
    assert benches_to_best([2, 0, 1], [1.0, None, 3.0]) == 1
    assert benches_to_best([0, 1], [None, None]) is None
    assert expected_random_benches(7) == 4.0
    assert abs(spearman([1, 2, 3], [3, 2, 1]) + 1) < 1e-12


def test_features_read_cuda_and_triton_and_task_context():
    from kore_b200.value.features import FEATURE_NAMES, featurize, schedule_features, task_features, tensor_core_tier
    cu = ("__global__ void __launch_bounds__(192, 1) k(...) {\n  constexpr int BM = 128;\n"
          "  __shared__ float red[32];\n  asm volatile(\"tcgen05.mma.cta_group::1.kind::f16 ...\");\n"
          "  asm volatile(\"cp.async.bulk.tensor.2d ...\");\n#pragma unroll\n  for (int i = 0; i < 4; ++i) {}\n"
          "  uint4 u = *p; v = __shfl_xor_sync(0xffffffff, v, 1);\n}")
    f = schedule_features(cu)
    assert f["tc_tcgen05"] == 1.0 and f["tma"] == 1.0 and f["log2_threads"] == pytest.approx(math.log2(192))
    assert f["log2_max_tile"] == 7.0 and f["vec16"] == 1.0 and f["shuffles"] > 0 and f["unroll"] > 0
    assert tensor_core_tier("wmma::mma_sync(c, a, b, c)") == "wmma"
    assert tensor_core_tier("asm(\"mma.sync.aligned.m16n8k16\")") == "mma_sync"
    tri = "BLOCK_M: tl.constexpr = 128\nnum_warps = 8\nacc = tl.zeros((BLOCK_M, BLOCK_N), dtype=tl.float32)\n"
    g = schedule_features(tri)
    assert g["log2_block_m"] == 7.0 and g["log2_num_warps"] == 3.0 and g["fp32_acc"] == 1.0
    t = task_features({"dtype": "bfloat16", "operation": "gemm_fused", "dims": {"M": 4096, "N": 4096, "K": 1024},
                       "intensity": 1000.0, "bound": "compute"})
    assert t["dtype_bf16"] == 1.0 and t["op_gemm"] == 1.0 and t["log2_dim0"] > 11.9 and t["memory_bound"] == 0.0
    assert task_features({"operation": "rmsnorm_bwd"})["op_train"] == 1.0
    v = featurize(cu, {"dtype": "fp8", "operation": "attention_decode"})
    assert v.shape == (len(FEATURE_NAMES),) and v[-1] == 1.0


def test_v2_model_learns_synthetic_ground_truth_and_roundtrips():
    from kore_b200.value.features import synthesize_groups
    from kore_b200.value.model import ValueModel, refit_online
    from kore_b200.value.rerank import groupwise_spearman, score_candidates, top_k_recall
    train, held = synthesize_groups(300, seed=1), synthesize_groups(60, seed=2)
    m = ValueModel().fit_groups(train)

    def score(rows):
        return list(m.predict(m.featurize([r["source"] for r in rows], rows[0]["meta"]))["rank_score"])
    rho = groupwise_spearman(score, held)
    assert rho > 0.4, rho
    rec = [top_k_recall(score(g), [r["speedup"] for r in g], 2) for g in held]
    rec = [x for x in rec if x == x]
    assert sum(rec) / len(rec) > 0.5
    m2 = ValueModel.from_json(m.to_json())
    assert m2.featurizer == "v2"
    srcs = [r["source"] for r in held[0]]
    assert score_candidates(srcs, model=m2) == score_candidates(srcs, model=m)
    buf = []
    m3 = refit_online(buf, train[:50], max_groups=40)
    assert len(buf) == 40 and m3.w_rank is not None


def test_v1_models_still_load():
    import json

    from kore_b200.value.model import ValueModel, features
    F = np.stack([features("BM = %d\nnum_warps = 4" % b) for b in (32, 64, 128, 256)])
    m = ValueModel("v1").fit(F, np.ones(4, bool), np.ones(4, bool), np.log([1.0, 1.5, 2.0, 1.2]))
    d = json.loads(m.to_json())
    d.pop("featurizer")                                   # a file written before the field existed
    old = ValueModel.from_json(json.dumps(d))
    assert old.featurizer == "v1" and old.featurize(["BM = 64"]).shape == (1, F.shape[1])
