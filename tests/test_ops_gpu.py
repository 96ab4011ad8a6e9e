"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

from kore_b200 import ops
from kore_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 192), (1000, 1536, 640),
                                   (4096, 7168, 5120), (264, 136, 72), (8, 128, 4096)])
@pytest.mark.parametrize("a_t,b_t", [(False, True), (False, False), (True, False), (True, True)])
def test_gemm_layouts(M, N, K, a_t, b_t):
    torch.manual_seed(0)
    A = torch.randn(K, M) if a_t else torch.randn(M, K)
    B = torch.randn(N, K) if b_t else torch.randn(K, N)
    A = A.cuda().bfloat16()
    B = B.cuda().bfloat16()
    out = ops.mm(A, B, a_t=a_t, b_t=b_t)
    Af = A.float().t() if a_t else A.float()
    Bf = B.float().t() if b_t else B.float()
    want = Af @ Bf
    assert ops.check_device_error() == 0
    assert _rel(out, want) < 8e-3


def test_gemm_epilogues():
    torch.manual_seed(1)
    M, N, K = 512, 768, 256
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    R = torch.randn(M, N, device="cuda").bfloat16()
    want = A.float() @ B.float().t()
    out = ops.mm(A, B, residual=R)
    assert _rel(out, want + R.float()) < 8e-3
    acc = torch.randn(M, N, device="cuda")
    acc0 = acc.clone()
    ops.mm(A, B, out=acc, accumulate=True, alpha=0.5)
    assert _rel(acc, acc0 + 0.5 * want) < 5e-3
    o32 = ops.mm(A, B, out_dtype=torch.float32)
    assert _rel(o32, want) < 1e-5 * 0 + 2e-3
    assert ops.check_device_error() == 0


@pytest.mark.parametrize("M,N,K", [(8192, 7168, 512), (4000, 5120, 1024), (5120, 34816, 256),
                                   (1000, 9536, 512), (4200, 5120, 256)])
@pytest.mark.parametrize("a_t,b_t", [(False, True), (False, False), (True, False), (True, True)])
def test_gemm_pair_kernel(M, N, K, a_t, b_t):
    """2-CTA (cta_group::2) kernel: every operand layout, ragged M and N
    (including last tiles where the second CTA's rows or columns lie wholly
    past the matrix)."""
    C = ops.native()
    torch.manual_seed(5)
    A = (torch.randn(K, M) if a_t else torch.randn(M, K)).cuda().bfloat16()
    B = (torch.randn(N, K) if b_t else torch.randn(K, N)).cuda().bfloat16()
    R = torch.randn(M, N, device="cuda").bfloat16()
    old = C.gemm_set_pair_mode(1)
    try:
        out = ops.mm(A, B, a_t=a_t, b_t=b_t, residual=R)
        o32 = ops.mm(A, B, a_t=a_t, b_t=b_t, out_dtype=torch.float32)
    finally:
        C.gemm_set_pair_mode(old)
    Af = A.float().t() if a_t else A.float()
    Bf = B.float().t() if b_t else B.float()
    want = Af @ Bf
    assert ops.check_device_error() == 0
    assert _rel(out, want + R.float()) < 8e-3
    assert _rel(o32, want) < 2e-3


@pytest.mark.parametrize("M,N,K", [(64, 7168, 5120), (1, 5120, 17408), (200, 1024, 4096)])
def test_gemm_split_k_epilogues(M, N, K):
    """Skinny (decode-sized) GEMMs split K over the SMs; the reduce applies
    alpha, the residual and accumulation."""
    torch.manual_seed(2)
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") / math.sqrt(K)).bfloat16()
    R = torch.randn(M, N, device="cuda").bfloat16()
    want = A.float() @ B.float().t()
    assert _rel(ops.mm(A, B), want) < 8e-3
    assert _rel(ops.mm(A, B, residual=R), want + R.float()) < 8e-3
    acc = torch.randn(M, N, device="cuda")
    acc0 = acc.clone()
    ops.mm(A, B, out=acc, accumulate=True, alpha=0.5)
    assert _rel(acc, acc0 + 0.5 * want) < 5e-3
    accb = torch.randn(M, N, device="cuda").bfloat16()
    accb0 = accb.float().clone()
    ops.mm(A, B, out=accb, accumulate=True)
    assert _rel(accb, accb0 + want) < 8e-3
    assert ops.check_device_error() == 0


@pytest.mark.parametrize("T,H,with_res", [(300, 5120, True), (4099, 5120, False), (1500, 2048, True),
                                           (777, 8192, True), (2000, 1024, False)])
def test_rmsnorm_fwd_bwd(T, H, with_res):
    """Row counts above and below the persistent grid (so blocks walk several
    rows with the next row prefetched), every vector-per-thread instantiation,
    with and without the residual gradient."""
    torch.manual_seed(2)
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    rstd = torch.empty(T, device="cuda")
    y = ops.rmsnorm_fwd(x, w, 1e-6, rstd=rstd)
    assert _rel(y, ref.rmsnorm(x.float(), w.float(), 1e-6)) < 5e-3
    dy = torch.randn(T, H, device="cuda").bfloat16()
    dres = torch.randn(T, H, device="cuda").bfloat16() if with_res else None
    dw = torch.zeros(H, device="cuda")
    dx = ops.rmsnorm_bwd(dy, x, w, rstd, dres=dres, dw=dw)
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    yr = ref.rmsnorm(xf, wf, 1e-6)
    yr.backward(dy.float())
    assert _rel(dx, xf.grad + (dres.float() if with_res else 0.0)) < 8e-3
    assert _rel(dw, wf.grad) < 5e-3


def test_qk_norm_rope():
    torch.manual_seed(3)
    T, hq, hkv, D = 257, 8, 2, 128
    qkv = torch.randn(T, (hq + 2 * hkv) * D, device="cuda").bfloat16()
    qw = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
    pos = torch.randint(0, 4096, (T,), device="cuda", dtype=torch.int32)
    cos, sin = ref.rope_tables(4096, D, 1e6, "cuda")
    out = ops.qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, hq, hkv, 1e-6)
    want = ref.qk_norm_rope(qkv.float(), qw.float(), kw.float(), pos, cos, sin, hq, hkv, 1e-6)
    assert _rel(out, want) < 5e-3
    dout = torch.randn_like(out)
    dqkv = torch.zeros_like(qkv)
    dqw = torch.zeros(D, device="cuda")
    dkw = torch.zeros(D, device="cuda")
    ops.qk_norm_rope_bwd(dout, qkv, qw, kw, pos, cos, sin, dqkv, dqw, dkw, hq, hkv, 1e-6)
    x = qkv.float().requires_grad_(True)
    qwf = qw.float().requires_grad_(True)
    kwf = kw.float().requires_grad_(True)
    ref.qk_norm_rope(x, qwf, kwf, pos, cos, sin, hq, hkv, 1e-6).backward(dout.float())
    n = (hq + hkv) * D
    assert _rel(dqkv[:, :n], x.grad[:, :n]) < 8e-3
    assert _rel(dqw, qwf.grad) < 5e-3 and _rel(dkw, kwf.grad) < 5e-3


def test_swiglu():
    torch.manual_seed(4)
    gu = torch.randn(333, 2 * 704, device="cuda").bfloat16()
    out = ops.swiglu_fwd(gu)
    assert _rel(out, ref.swiglu(gu.float())) < 5e-3
    d = torch.randn_like(out)
    x = gu.float().requires_grad_(True)
    ref.swiglu(x).backward(d.float())
    dgu = ops.swiglu_bwd(d, gu)
    assert _rel(dgu, x.grad) < 8e-3


@pytest.mark.parametrize("V,temp", [(151936, 1.0), (32000, 0.7)])
def test_logprob_and_grad(V, temp):
    torch.manual_seed(5)
    T = 64
    logits = (3 * torch.randn(T, V, device="cuda")).bfloat16()
    tg = torch.randint(0, V, (T,), device="cuda")
    lp, ent, lse = ops.logprob(logits, tg, temp, want_entropy=True, want_lse=True)
    a, b, c = ref.token_logprobs(logits.float(), tg, temp)
    assert torch.allclose(lp, a, atol=2e-3, rtol=1e-4)
    assert torch.allclose(ent, b, atol=2e-3, rtol=1e-4)
    coef = torch.randn(T, device="cuda")
    z = logits.float().requires_grad_(True)
    la, _, _ = ref.token_logprobs(z, tg, temp)
    (la * coef).sum().backward()
    g = logits.clone()
    ops.logprob(g, tg, temp, coef=coef, write_grad=True)
    assert _rel(g, z.grad) < 1e-2


def test_adamw_matches_torch():
    torch.manual_seed(6)
    n = 100_003
    p32 = torch.randn(n, device="cuda")
    p = p32.bfloat16()
    master = p.float().clone()
    g = torch.randn(n, device="cuda").bfloat16()
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    tp = torch.nn.Parameter(master.clone())
    opt = torch.optim.AdamW([tp], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(1, 4):
        tp.grad = g.float().clone()
        opt.step()
        ops.adamw_step(p, g, m, v, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, step=step,
                       master=master)
    assert torch.allclose(master, tp.detach(), atol=1e-6, rtol=1e-5)


def test_sumsq_and_clip():
    g = torch.randn(1 << 20, device="cuda").bfloat16()
    s = torch.zeros(1, device="cuda")
    ops.sumsq(g, s)
    assert math.isclose(s.item(), g.float().pow(2).sum().item(), rel_tol=1e-4)


@pytest.mark.parametrize("use_master", [True, False])
def test_adamw_vectorized_path_matches_torch(use_master):
    """n % 8 == 0 takes the 16-byte vectorised kernel; without a master copy the
    bf16 write is stochastically rounded (within one bf16 ulp of fp32 AdamW)."""
    torch.manual_seed(7)
    n = 1 << 20
    p = torch.randn(n, device="cuda").bfloat16()
    master = p.float().clone()
    g = torch.randn(n, device="cuda").bfloat16()
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    tp = torch.nn.Parameter(p.float().clone())
    opt = torch.optim.AdamW([tp], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    tp.grad = g.float().clone()
    opt.step()
    ops.adamw_step(p, g, m, v, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, step=1,
                   master=master if use_master else None)
    if use_master:
        assert torch.allclose(master, tp.detach(), atol=1e-6, rtol=1e-5)
    ulp = tp.detach().abs() * 2 ** -7 + 1e-30
    assert ((p.float() - tp.detach()).abs() <= ulp).all()
