"""MoE ops: router, permutation, grouped expert GEMM, combine.

CUDA tensors run the native kernels (tcgen05 grouped GEMM, routing and
combine kernels); CPU tensors run the PyTorch definitions below (tests and
gloo runs)."""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from . import embed_fwd
from ._lib import native


def route(logits: torch.Tensor, k: int, norm: bool = True):
    """softmax over experts -> top-k -> optional renormalisation.
    Returns (probs [T,E] fp32, idx [T,k] int32, w [T,k] fp32)."""
    T, E = logits.shape
    if logits.is_cuda:
        probs = torch.empty(T, E, dtype=torch.float32, device=logits.device)
        idx = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        native().moe_route_fwd(logits.float().contiguous(), k, bool(norm), probs, idx, w)
        return probs, idx, w
    probs = torch.softmax(logits.float(), -1)
    w, idx = probs.topk(k, -1)
    if norm:
        w = w / w.sum(-1, keepdim=True)
    return probs, idx.int(), w


def route_bwd(probs, idx, w, dw, norm: bool = True):
    if probs.is_cuda:
        out = torch.empty_like(probs)
        native().moe_route_bwd(probs, idx, w, dw.float().contiguous(), bool(norm), out)
        return out
    p = probs.detach().requires_grad_(True)
    with torch.enable_grad():
        sel = p.gather(-1, idx.long())
        ww = sel / sel.sum(-1, keepdim=True) if norm else sel
        # d logits = softmax bwd of d probs
        gp, = torch.autograd.grad(ww, p, dw)
    return probs * (gp - (gp * probs).sum(-1, keepdim=True))


def permutation(idx: torch.Tensor, num_experts: int, expert_range: Optional[Tuple[int, int]] = None):
    """Expert-major ordering of the (token, slot) pairs.

    Returns (src_token [P] long: token of each permuted row, pos [T,k] int32:
    permuted row of each pair or -1 when the expert is outside
    ``expert_range``, offsets: host list of E_local+1 row offsets)."""
    T, k = idx.shape
    flat = idx.reshape(-1).long()
    lo, hi = expert_range if expert_range is not None else (0, num_experts)
    keep = (flat >= lo) & (flat < hi)
    order = torch.argsort(torch.where(keep, flat, torch.full_like(flat, hi)), stable=True)
    n_keep = int(keep.sum())
    order = order[:n_keep]
    counts = torch.bincount(flat[keep] - lo, minlength=hi - lo).tolist()
    offsets = [0]
    for c in counts:
        offsets.append(offsets[-1] + int(c))
    pos = torch.full((T * k,), -1, dtype=torch.int32, device=idx.device)
    pos[order] = torch.arange(n_keep, dtype=torch.int32, device=idx.device)
    return order // k, pos.view(T, k), offsets


def gather_rows(x: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    return embed_fwd(rows, x)


def grouped_mm(a: torch.Tensor, w: torch.Tensor, offsets: List[int], *, w_t: bool = True,
               out: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    """Per expert e: out[rows_e] = a[rows_e] @ (w[e].T if w_t else w[e]).
    w: [E, N, K] when w_t else [E, K, N]."""
    N = w.shape[1] if w_t else w.shape[2]
    if out is None:
        out = torch.empty(a.shape[0], N, dtype=a.dtype, device=a.device)
    if a.is_cuda:
        native().gemm_grouped_bf16(a, w, out, [int(o) for o in offsets], not w_t, bool(accumulate))
        return out
    for e in range(len(offsets) - 1):
        s, t = offsets[e], offsets[e + 1]
        if t > s:
            r = a[s:t].float() @ (w[e].float().t() if w_t else w[e].float())
            out[s:t] = (r + out[s:t].float() if accumulate else r).to(out.dtype)
    return out


def combine(src, pos, w=None, resid=None, out=None):
    T, k = pos.shape
    H = src.shape[1]
    if out is None:
        out = torch.empty(T, H, dtype=src.dtype, device=src.device)
    if src.is_cuda:
        native().moe_combine(src, pos, w.float().contiguous() if w is not None else None, resid, out)
        return out
    acc = resid.float().clone() if resid is not None else torch.zeros(T, H, device=src.device)
    valid = pos >= 0
    g = src.float()[pos.clamp_min(0).long()]                       # [T,k,H]
    ww = (w.float() if w is not None else torch.ones(T, k, device=src.device)) * valid
    out.copy_((acc + (g * ww.unsqueeze(-1)).sum(1)).to(out.dtype))
    return out


def combine_bwd(dy, src, pos, w):
    T, k = pos.shape
    dsrc = torch.zeros_like(src)
    if src.is_cuda:
        dw = torch.empty(T, k, dtype=torch.float32, device=src.device)
        native().moe_combine_bwd(dy, src, pos, w.float().contiguous(), dsrc, dw)
        return dsrc, dw
    valid = (pos >= 0)
    p = pos.clamp_min(0).long()
    dw = (dy.float().unsqueeze(1) * src.float()[p]).sum(-1) * valid
    contrib = (w.float() * valid).unsqueeze(-1) * dy.float().unsqueeze(1)    # [T,k,H]
    dsrc.index_put_((p[valid],), contrib[valid].to(src.dtype), accumulate=True)
    return dsrc, dw


# ----------------------------------------------------------------------------- device plan
PAD = 64


class Plan:
    """Expert-major routing plan with every expert's rows padded to a multiple
    of 64 (pad rows are zero). All fields stay on the device on CUDA: the
    grouped GEMMs read the tile table and row offsets there, so a MoE layer
    needs no host synchronisation.

    pos [T, k] int32: padded row of each (token, slot) pair (-1 outside the
    local experts); src_row [R] int32: source token of each row (-1 = pad);
    offsets [E_local + 1] int32; tiles [cap, 4] int32 / ntiles [1] int32: the
    grouped GEMM's 128-row tiles; R: row capacity (T k + E_local 63)."""

    def __init__(self, pos, src_row, offsets, tiles, ntiles, counts, rows: int):
        self.pos, self.src_row, self.offsets = pos, src_row, offsets
        self.tiles, self.ntiles, self.counts, self.rows = tiles, ntiles, counts, rows


def plan(idx: torch.Tensor, num_experts: int, expert_range: Optional[Tuple[int, int]] = None) -> Plan:
    T, k = idx.shape
    lo, hi = expert_range if expert_range is not None else (0, num_experts)
    El = hi - lo
    R = T * k + El * (PAD - 1)
    cap = R // 128 + El
    dev = idx.device
    i32 = dict(dtype=torch.int32, device=dev)
    pos = torch.empty(T * k, **i32)
    src_row = torch.empty(R, **i32)
    offsets = torch.empty(El + 1, **i32)
    tiles = torch.zeros(cap * 4, **i32)
    ntiles = torch.zeros(1, **i32)
    counts = torch.empty(El, **i32)
    if idx.is_cuda:
        native().moe_plan(idx.int().contiguous(), lo, hi, pos, src_row, offsets, tiles, ntiles, counts)
        return Plan(pos.view(T, k), src_row, offsets, tiles, ntiles, counts, R)
    # CPU definition (same layout)
    flat = idx.reshape(-1).long()
    pos.fill_(-1)
    src_row.fill_(-1)
    off, t = 0, 0
    for j in range(El):
        hit = (flat == lo + j).nonzero().reshape(-1)
        c = hit.numel()
        pc = (c + PAD - 1) // PAD * PAD
        counts[j] = c
        offsets[j] = off
        pos[hit] = off + torch.arange(c, dtype=torch.int32)
        src_row[off:off + c] = (hit // k).int()
        for r in range(0, pc, 128):
            tiles[4 * t: 4 * t + 4] = torch.tensor([j, off + r, off + pc, 0], dtype=torch.int32)
            t += 1
        off += pc
    offsets[El] = off
    ntiles[0] = t
    return Plan(pos.view(T, k), src_row, offsets, tiles, ntiles, counts, R)


def plan_gather(x: torch.Tensor, p: Plan) -> torch.Tensor:
    """Rows of ``x`` in the plan's padded expert-major order (zero pad rows)."""
    out = torch.empty(p.rows, x.shape[1], dtype=x.dtype, device=x.device)
    if x.is_cuda:
        native().moe_gather_rows(x.contiguous(), p.src_row, out)
        return out
    valid = p.src_row >= 0
    out.zero_()
    out[valid] = x[p.src_row[valid].long()]
    return out


def plan_mm(a: torch.Tensor, w: torch.Tensor, p: Plan, *, w_t: bool = True,
            out: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    """Per expert e: rows of e (padded block) = a_e @ (w[e].T if w_t else w[e])."""
    N = w.shape[1] if w_t else w.shape[2]
    if out is None:
        out = torch.zeros(a.shape[0], N, dtype=a.dtype, device=a.device) if not a.is_cuda else \
            torch.empty(a.shape[0], N, dtype=a.dtype, device=a.device)
    if a.is_cuda:
        native().gemm_grouped_dev(a, w, out, p.tiles, p.ntiles, not w_t, bool(accumulate))
        return out
    offs = p.offsets.tolist()
    for e in range(len(offs) - 1):
        s, t = offs[e], offs[e + 1]
        if t > s:
            r = a[s:t].float() @ (w[e].float().t() if w_t else w[e].float())
            out[s:t] = (r + out[s:t].float() if accumulate else r).to(out.dtype)
    return out


def plan_wgrad(dy: torch.Tensor, x: torch.Tensor, p: Plan, out: torch.Tensor, accumulate: bool = True) -> None:
    """out[e] (+)= dy[rows_e]^T x[rows_e] for every local expert, one launch."""
    if dy.is_cuda:
        native().gemm_grouped_wgrad(dy.contiguous(), x.contiguous(), out, p.offsets, bool(accumulate))
        return
    offs = p.offsets.tolist()
    for e in range(len(offs) - 1):
        s, t = offs[e], offs[e + 1]
        if t > s:
            r = dy[s:t].float().t() @ x[s:t].float()
            out[e] = (r + out[e].float() if accumulate else r).to(out.dtype)
