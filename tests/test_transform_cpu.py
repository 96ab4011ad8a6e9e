"""Transform calculus: relation typing, epsilon lattice and budget, the
admissible action space (monotone in the budget), audited trajectories, the
per-family rewrites and the opt-in discovered families."""
import pytest

from kore_b200.transform import (APPROX, EXACT, ErrorBudget, LIBRARY, admissible, apply_sequence,
                                 compose_eps, compose_relation, default_epsilon, get_transform)
from kore_b200.transform.calculus import admissible_actions
from kore_b200.transform.discover import discover_transforms, extend_library

GEMM = '''import torch
import triton
import triton.language as tl


@triton.jit
def _k(A, B, C, M, N, K, BM: tl.constexpr, BN: tl.constexpr, BK: tl.constexpr, GROUP_M: tl.constexpr):
    pm, pn = tl.program_id(0), tl.program_id(1)
    rm = pm * BM + tl.arange(0, BM)
    rn = pn * BN + tl.arange(0, BN)
    rk = tl.arange(0, BK)
    acc = tl.zeros((BM, BN), dtype=tl.float16)
    for k in range(0, K, BK):
        a = tl.load(A + rm[:, None] * K + (k + rk)[None, :])
        b = tl.load(B + rn[None, :] * K + (k + rk)[:, None])
        acc += tl.dot(a, b)
    tl.store(C + rm[:, None] * N + rn[None, :], acc.to(C.dtype.element_ty))


def gemm(a, b):
    M, K = a.shape
    N = b.shape[0]
    c = torch.empty(M, N, device=a.device, dtype=a.dtype)
    _k[(triton.cdiv(M, 64), triton.cdiv(N, 64))](a, b, c, M, N, K, BM=64, BN=64, BK=32, GROUP_M=8)
    return c
'''

NORM = '''import torch
import triton
import triton.language as tl


@triton.jit
def _k(X, Y, N, eps, BLOCK: tl.constexpr, VEC: tl.constexpr):
    row = tl.program_id(0)
    cols = tl.arange(0, BLOCK)
    m = cols < N
    x = tl.load(X + row * N + cols, mask=m, other=0.0).to(tl.float32)
    r = 1.0 / tl.sqrt(tl.sum(x * x, 0) / N + eps)
    y = x * r
    tl.store(Y + row * N + cols, y, mask=m)


def norm(x):
    y = torch.empty_like(x)
    _k[(x.shape[0],)](x, y, x.shape[1], 1e-6, BLOCK=1024, VEC=4)
    return y
'''


def test_relation_lattice_and_budget():
    assert compose_relation(EXACT, EXACT) == EXACT
    assert compose_relation(EXACT, APPROX) == APPROX == compose_relation(APPROX, EXACT)
    assert compose_eps(0.01, 0.03) == 0.03
    with pytest.raises(ValueError):
        compose_relation("maybe", EXACT)
    assert default_epsilon("gemm", "bf16") < default_epsilon("gelu", "bf16")
    assert default_epsilon("gemm", "fp32") < default_epsilon("gemm", "bf16") < default_epsilon("gemm", "fp8")
    b = ErrorBudget(total=0.05)
    b.spend("a", APPROX, 0.03)
    b.spend("b", EXACT, 0.0)
    assert abs(b.remaining() - 0.02) < 1e-12 and b.composed_relation() == APPROX and b.weakest_eps() == 0.03
    assert not b.affords(APPROX, 0.03) and b.affords(EXACT, 10.0)
    with pytest.raises(ValueError):
        b.spend("c", APPROX, 0.05)


def test_every_family_is_typed_and_exact_ones_are_exact():
    names = {t.name for t in LIBRARY}
    assert len(LIBRARY) >= 16 and len(names) == len(LIBRARY)
    for t in LIBRARY:
        assert t.kind in (EXACT, APPROX)
        for a in t.actions(GEMM) + t.actions(NORM):
            assert (a.eps == 0.0) == (t.kind == EXACT)


def test_action_space_is_monotone_in_budget():
    big = {a.name for a in admissible_actions(GEMM, budget=ErrorBudget(total=1.0))}
    small = {a.name for a in admissible_actions(GEMM, budget=ErrorBudget(total=0.01))}
    none = {a.name for a in admissible_actions(GEMM, budget=ErrorBudget(total=0.0))}
    assert none <= small <= big and len(none) < len(big)
    assert all(get_transform(n.split("(")[0]).kind == EXACT for n in none)


def test_gemm_rewrites():
    out = get_transform("split_k(ways=4)").apply(GEMM)
    assert "tl.atomic_add(" in out and "SPLIT_K=4" in out and "torch.zeros(" in out
    assert "range(tl.program_id(2) * BK, K, BK * SPLIT_K)" in out and ", 4)](" in out
    assert "dtype=tl.float32" in get_transform("fp32_accumulator").apply(GEMM)
    assert "acc = tl.dot(a, b, acc)" in get_transform("reassociate_reduction").apply(GEMM)
    assert "a.to(tl.float8e4nv)" in get_transform("downcast_dtype(to=fp8)").apply(GEMM)
    assert "warp_specialize=True" in get_transform("warp_specialize").apply(GEMM)
    assert "GROUP_M=16" in get_transform("swizzle_group_m(g=16)").apply(GEMM)
    assert "num_ctas=2" in get_transform("set_num_ctas(n=2)").apply(GEMM)
    assert "num_stages=4" in get_transform("set_num_stages(n=4)").apply(GEMM)
    swapped = get_transform("reorder_loads").apply(GEMM)
    assert swapped.index("b = tl.load") < swapped.index("a = tl.load")


def test_norm_rewrites_and_side_conditions():
    assert "tl.rsqrt(" in get_transform("rsqrt").apply(NORM)
    assert "tl.multiple_of(cols, 16)" in get_transform("vectorize_loads(width=16)").apply(NORM)
    assert get_transform("split_k").apply(NORM) is None              # no K loop: does not apply
    assert "BLOCK=512" in get_transform("retile_block(f=half,name=BLOCK)").apply(NORM)
    biased = GEMM.replace("acc.to(C.dtype.element_ty))", "acc.to(C.dtype.element_ty) + bias)")
    _, applied, rejected, state = apply_sequence(biased, [("split_k", {"ways": 2})], ErrorBudget(1.0), audit=True)
    assert not applied and "side condition" in rejected[0].reason


def test_audited_trajectory_and_budget_refusal():
    steps = [("set_num_stages", {"n": 4}), ("downcast_dtype", {"to": "fp8"}), ("reassociate_reduction", {}),
             ("no_such_transform", {})]
    out, applied, rejected, state = apply_sequence(GEMM, steps, ErrorBudget(total=0.05), audit=True)
    assert [r.name for r in applied] == ["set_num_stages(n=4)", "reassociate_reduction"]
    reasons = {r.name: r.reason for r in rejected}
    assert reasons["downcast_dtype(to=fp8)"].startswith("budget") and "unknown" in reasons["('no_such_transform', {})"]
    assert state["relation"] == APPROX and abs(state["spent"] - 0.01) < 1e-12


def test_discovered_families_are_opt_in_and_approx():
    src = NORM.replace("VEC=4", "VEC=4").replace("cols = tl.arange(0, BLOCK)\n",
                                               "cols = tl.arange(0, BLOCK)\n    cols = tl.max_contiguous(tl.multiple_of(cols, 16), 16)\n")
    found = discover_transforms(src)
    names = {t.name for t in found}
    assert "sweep_vec" in names and "discovered_vector_width" in names and "fuse_epilogue" in names
    assert all(t.kind == APPROX and t.epsilon({}) > 0 for t in found)
    assert extend_library(src) == list(LIBRARY)
    ext = extend_library(src, enabled=True)
    assert len(ext) == len(LIBRARY) + len(found)
    fused = [t for t in found if t.name == "fuse_epilogue"][0].apply(src)
    assert "tl.store(Y + row * N + cols, (x * r), mask=m)" in fused


CUDA_SRC = '''__global__ void scale(const float* x, float* y, int n) {
  for (int i = 0; i < 4; ++i) { y[i] = x[i]; }
}
void run(const float* x, float* y, int n) { scale<<<n / 256, 256>>>(x, y, n); }
'''


def test_cuda_rewrite_families():
    from kore_b200.transform.library import EXACT_LIBRARY, get_transform
    names = {t.name for t in EXACT_LIBRARY}
    assert {"cuda_launch_bounds", "cuda_restrict", "cuda_unroll"} <= names
    lb = get_transform("cuda_launch_bounds")
    assert lb.domain(CUDA_SRC)[0] == {"threads": 256, "min_blocks": 1}
    out = lb.apply(CUDA_SRC)
    assert "__launch_bounds__(256, 1) void scale" in out
    assert "__launch_bounds__(512, 2)" in lb.apply(out, threads=512, min_blocks=2)      # replaces, not stacks
    assert lb.apply(CUDA_SRC, threads=128, min_blocks=1) is None                          # launch uses 256
    r = get_transform("cuda_restrict").apply(CUDA_SRC)
    assert "const float* __restrict__ x, float* __restrict__ y, int n" in r
    assert get_transform("cuda_restrict").apply(CUDA_SRC.replace("(x, y, n)", "(x, x, n)")) is None
    u = get_transform("cuda_unroll").apply(CUDA_SRC)
    assert "#pragma unroll\n  for (int i = 0; i < 4" in u and get_transform("cuda_unroll").apply(u) is None
    assert get_transform("cuda_unroll").apply("def f(x):\n    return x\n") is None
