"""Causal GQA attention over packed (varlen) sequences.

Layout: q [T, Hq, D], k/v [T, Hkv, D] (strided views are fine), sequence
boundaries ``cu_seqlens`` (int32, [n+1]). Forward returns o [T, Hq, D] and
the per-row logsumexp lse [Hq, T] (fp32) needed by the backward.

CUDA tensors always run the native sm_100a kernels (``_C.attn_fwd`` /
``_C.attn_bwd``); if the extension is missing the call raises, there is no
library fallback on a GPU. CPU tensors use the fp32 PyTorch definition.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import reference as ref
from ._lib import native


def _seq_bounds(cu_seqlens: Optional[torch.Tensor], T: int):
    if cu_seqlens is None:
        return [(0, T)]
    cu = [int(c) for c in cu_seqlens.tolist()]
    return list(zip(cu[:-1], cu[1:]))


def attn_fwd(q, k, v, cu_seqlens=None, max_seqlen: int = 0, scale: Optional[float] = None
             ) -> Tuple[torch.Tensor, torch.Tensor]:
    T, hq, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if q.is_cuda:
        o = torch.empty(T, hq, D, dtype=q.dtype, device=q.device)
        lse = torch.empty(hq, T, dtype=torch.float32, device=q.device)
        cu = cu_seqlens if cu_seqlens is not None else torch.tensor([0, T], dtype=torch.int32, device=q.device)
        native().attn_fwd(q, k, v, cu, int(max_seqlen or T), float(scale), o, lse)
        return o, lse
    return _attn_fwd_torch(q, k, v, cu_seqlens, scale)


def attn_bwd(do, q, k, v, o, lse, cu_seqlens=None, max_seqlen: int = 0,
             scale: Optional[float] = None, dq=None, dk=None, dv=None):
    T, hq, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    dq = dq if dq is not None else torch.empty_like(q)
    dk = dk if dk is not None else torch.empty(k.shape, dtype=k.dtype, device=k.device)
    dv = dv if dv is not None else torch.empty(v.shape, dtype=v.dtype, device=v.device)
    if q.is_cuda:
        cu = cu_seqlens if cu_seqlens is not None else torch.tensor([0, T], dtype=torch.int32, device=q.device)
        # fp32 dQ accumulator and per-row delta: scratch of this call
        dq_acc = torch.empty(T, hq, D, dtype=torch.float32, device=q.device)
        delta = torch.empty(hq, T, dtype=torch.float32, device=q.device)
        native().attn_bwd(do, q, k, v, o.reshape(T, hq, D), lse, cu, int(max_seqlen or T),
                          float(scale), dq, dk, dv, dq_acc, delta)
        return dq, dk, dv
    with torch.enable_grad():
        qq = q.detach().requires_grad_(True)
        kk = k.detach().requires_grad_(True)
        vv = v.detach().requires_grad_(True)
        oo, _ = _attn_fwd_torch(qq, kk, vv, cu_seqlens, scale, need_lse=False)
        gq, gk, gv = torch.autograd.grad(oo, (qq, kk, vv), do)
    dq.copy_(gq)
    dk.copy_(gk)
    dv.copy_(gv)
    return dq, dk, dv


def _attn_fwd_torch(q, k, v, cu_seqlens, scale, need_lse: bool = True):
    """Plain fp32 PyTorch definition (CPU only; the reference the kernels are tested against)."""
    if q.is_cuda:
        raise RuntimeError("attention on CUDA tensors runs only on the native kernels")
    T, hq, D = q.shape
    hkv = k.shape[1]
    outs = []
    lses = []
    for a, b in _seq_bounds(cu_seqlens, T):
        qs = q[a:b].transpose(0, 1).unsqueeze(0)
        ks = k[a:b].transpose(0, 1).unsqueeze(0)
        vs = v[a:b].transpose(0, 1).unsqueeze(0)
        rep = hq // hkv
        kf = ks.float().repeat_interleave(rep, 1)
        vf = vs.float().repeat_interleave(rep, 1)
        s = (qs.float() @ kf.transpose(-1, -2)) * scale
        n = b - a
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
        o = (s.softmax(-1) @ vf).to(q.dtype)
        outs.append(o[0].transpose(0, 1))
        if need_lse:
            with torch.no_grad():
                rep = hq // hkv
                kf = ks.float().repeat_interleave(rep, 1)
                s = (qs.float() @ kf.transpose(-1, -2)) * scale
                n = b - a
                mask = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
                lses.append(torch.logsumexp(s.masked_fill(~mask, float("-inf")), -1)[0])
    o = torch.cat(outs, 0) if len(outs) > 1 else outs[0]
    lse = torch.cat(lses, 1) if (need_lse and lses) else None
    return o, lse
