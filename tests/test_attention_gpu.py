"""tcgen05 flash attention (fwd + bwd) against the fp32 PyTorch reference."""
import math

import pytest
import torch

from kore_b200.ops import attention as attn
from kore_b200.ops import native
from kore_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _inputs(lens, hq, hkv, seed=0):
    torch.manual_seed(seed)
    T = sum(lens)
    D = 128
    # q and k live in one fused buffer like the engine's (strided views)
    qk = torch.randn(T, (hq + hkv) * D, device="cuda").bfloat16()
    v = torch.randn(T, hkv * D, device="cuda").bfloat16()
    q = qk[:, : hq * D].view(T, hq, D)
    k = qk[:, hq * D:].view(T, hkv, D)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32,
                      device="cuda")
    return q, k, v.view(T, hkv, D), cu, max(lens)


@pytest.mark.parametrize("lens,hq,hkv", [([128], 2, 1), ([300], 4, 2), ([1000, 77, 256], 5, 1),
                                         ([2048], 8, 8)])
def test_attn_fwd(lens, hq, hkv):
    assert hasattr(native(), "attn_fwd")
    q, k, v, cu, mx = _inputs(lens, hq, hkv)
    o, lse = attn.attn_fwd(q, k, v, cu, mx)
    want = ref.causal_attention(q.float(), k.float(), v.float(), cu_seqlens=cu)
    assert _rel(o, want) < 1e-2
    # logsumexp of each row
    D = 128
    s0 = 0
    for n in lens:
        qs = q[s0:s0 + n].float().transpose(0, 1)
        ks = k[s0:s0 + n].float().repeat_interleave(hq // hkv, 1).transpose(0, 1)
        s = qs @ ks.transpose(-1, -2) / math.sqrt(D)
        s = s.masked_fill(~torch.ones(n, n, dtype=torch.bool, device="cuda").tril(), float("-inf"))
        assert torch.allclose(lse[:, s0:s0 + n], torch.logsumexp(s, -1), atol=2e-2)
        s0 += n


@pytest.mark.parametrize("lens,hq,hkv", [([128], 2, 1), ([300], 4, 2), ([700, 77, 256], 5, 1)])
def test_attn_bwd(lens, hq, hkv):
    q, k, v, cu, mx = _inputs(lens, hq, hkv, seed=1)
    o, lse = attn.attn_fwd(q, k, v, cu, mx)
    do = torch.randn_like(o)
    dq, dk, dv = attn.attn_bwd(do, q, k, v, o, lse, cu, mx)
    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    ref.causal_attention(qf, kf, vf, cu_seqlens=cu).backward(do.float())
    assert _rel(dq, qf.grad) < 2e-2
    assert _rel(dk, kf.grad) < 2e-2
    assert _rel(dv, vf.grad) < 2e-2
