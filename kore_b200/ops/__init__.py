"""Hot ops of kore_b200. CUDA tensors run the hand-written sm_100a kernels of
``kore_b200._C``; CPU tensors run the PyTorch definitions in
``kore_b200.ops.reference``."""
from __future__ import annotations

from typing import Optional

import torch

from . import reference as ref
from ._lib import available, check_device_error, launch_count, native, reset_launch_count

__all__ = [
    "available", "check_device_error", "native", "ref",
    "mm", "linear", "rmsnorm_fwd", "rmsnorm_bwd", "qk_norm_rope_fwd", "qk_norm_rope_bwd",
    "swiglu_fwd", "swiglu_bwd", "embed_fwd", "embed_bwd", "logprob", "sumsq", "adamw_step",
]


def mm(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = True,
       out: Optional[torch.Tensor] = None, alpha: float = 1.0, accumulate: bool = False,
       residual: Optional[torch.Tensor] = None, out_dtype=None) -> torch.Tensor:
    """out (=|+=) alpha * op(a) @ op(b) (+ residual).

    op(a) = a.T if a_t else a; op(b) = b.T if b_t else b.  With the defaults
    this is ``a @ b.T`` (a linear layer, weight [out, in]).  On CUDA this is
    the tcgen05 GEMM; transposed operands are read in place (MN-major UMMA).
    """
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[0] if b_t else b.shape[1]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype or a.dtype, device=a.device)
    if a.is_cuda:
        native().gemm_bf16(a, b, out, a_t, not b_t, float(alpha), bool(accumulate), residual, 0)
        return out
    A = a.t() if a_t else a
    B = b.t() if b_t else b
    r = (A.float() @ B.float()) * alpha
    if residual is not None:
        r = r + residual.float()
    if accumulate:
        r = r + out.float()
    out.copy_(r.to(out.dtype))
    return out


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None):
    """y = x @ w.T (+ residual), x [T, in], w [out, in]."""
    return mm(x, w, residual=residual)


def rmsnorm_fwd(x, w, eps, rstd: Optional[torch.Tensor] = None, out=None):
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        native().rmsnorm_fwd(x, w, out, rstd, float(eps))
        return out
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if rstd is not None:
        rstd.copy_(r.reshape(rstd.shape))
    out.copy_((xf * r * w.float()).to(x.dtype))
    return out


def rmsnorm_bwd(dy, x, w, rstd, dres=None, dw: Optional[torch.Tensor] = None, out=None):
    """dx = d rmsnorm(x)/dx . dy (+ dres); dw (fp32) += sum dy * xhat."""
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        native().rmsnorm_bwd(dy, x, w, rstd, dres, out, dw)
        return out
    H = x.shape[-1]
    r = rstd.reshape(-1, 1).float()
    xh = x.float().reshape(-1, H) * r
    g = dy.float().reshape(-1, H)
    if dw is not None:
        dw += (g * xh).sum(0)
    gw = g * w.float()
    dot = (gw * xh).mean(-1, keepdim=True)
    dx = r * (gw - xh * dot)
    if dres is not None:
        dx = dx + dres.float().reshape(-1, H)
    out.copy_(dx.reshape(x.shape).to(x.dtype))
    return out


def qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, hq, hkv, eps, rstd=None, out=None):
    T = qkv.shape[0]
    D = qkv.shape[1] // (hq + 2 * hkv)
    if out is None:
        out = torch.empty(T, (hq + hkv) * D, dtype=qkv.dtype, device=qkv.device)
    if qkv.is_cuda:
        native().qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, out, rstd, hq, hkv, float(eps))
        return out
    out.copy_(ref.qk_norm_rope(qkv, qw, kw, pos, cos, sin, hq, hkv, eps))
    return out


def qk_norm_rope_bwd(dout, qkv, qw, kw, pos, cos, sin, dqkv, dqw, dkw, hq, hkv, eps):
    """Writes d(raw q,k) into dqkv[:, :(hq+hkv)*D]; accumulates fp32 dqw/dkw."""
    if qkv.is_cuda:
        native().qk_norm_rope_bwd(dout, qkv, qw, kw, pos, cos, sin, dqkv, dqw, dkw, hq, hkv,
                                  float(eps))
        return dqkv
    T = qkv.shape[0]
    D = qkv.shape[1] // (hq + 2 * hkv)
    with torch.enable_grad():
        x = qkv[:, : (hq + hkv) * D].detach().float().requires_grad_(True)
        qwf = qw.detach().float().requires_grad_(True)
        kwf = kw.detach().float().requires_grad_(True)
        full = torch.cat([x, qkv[:, (hq + hkv) * D:].float()], 1)
        y = ref.qk_norm_rope(full, qwf, kwf, pos, cos, sin, hq, hkv, eps)
        y.backward(dout.float())
    dqkv[:, : (hq + hkv) * D].copy_(x.grad.to(dqkv.dtype))
    dqw += qwf.grad
    dkw += kwf.grad
    return dqkv


def swiglu_fwd(gu, out=None):
    F_ = gu.shape[1] // 2
    if out is None:
        out = torch.empty(gu.shape[0], F_, dtype=gu.dtype, device=gu.device)
    if gu.is_cuda:
        native().swiglu_fwd(gu, out)
        return out
    out.copy_(ref.swiglu(gu))
    return out


def swiglu_bwd(dout, gu, dgu=None):
    """d[gate|up]; dgu may alias gu (in place)."""
    if dgu is None:
        dgu = torch.empty_like(gu)
    if gu.is_cuda:
        native().swiglu_bwd(dout, gu, dgu)
        return dgu
    F_ = gu.shape[1] // 2
    g, u, d = gu[:, :F_].float(), gu[:, F_:].float(), dout.float()
    s = torch.sigmoid(g)
    dg = d * u * (s + g * s * (1 - s))
    du = d * g * s
    dgu[:, :F_].copy_(dg.to(dgu.dtype))
    dgu[:, F_:].copy_(du.to(dgu.dtype))
    return dgu


def embed_fwd(ids, table, out=None):
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    if table.is_cuda:
        native().embed_fwd(ids.reshape(-1), table, out)
        return out
    out.copy_(table[ids.reshape(-1)])
    return out


def embed_bwd(ids, dy, dtable):
    """dtable (fp32 or bf16) += scatter of dy rows by token id."""
    if dy.is_cuda:
        native().embed_bwd(ids.reshape(-1), dy, dtable)
        return dtable
    dtable.index_add_(0, ids.reshape(-1), dy.to(dtable.dtype))
    return dtable


def logprob(logits, targets=None, temperature: float = 1.0, *, want_entropy=False,
            want_lse=False, coef=None, write_grad=False):
    """Per-row log p(target), entropy and logsumexp of logits/temperature.

    With ``write_grad`` the bf16 ``logits`` buffer is overwritten in place by
    d(sum_t coef_t * logp_t)/d logits.  Returns (logp, entropy|None, lse|None).
    """
    T = logits.shape[0]
    dev = logits.device
    lp = torch.empty(T, dtype=torch.float32, device=dev) if targets is not None else None
    ent = torch.empty(T, dtype=torch.float32, device=dev) if want_entropy else None
    lse = torch.empty(T, dtype=torch.float32, device=dev) if want_lse else None
    inv_t = 1.0 / float(temperature)
    if logits.is_cuda:
        native().logprob_fwd_bwd(logits, targets, inv_t, lp, ent, lse,
                                 coef.float().contiguous() if coef is not None else None,
                                 bool(write_grad))
        return lp, ent, lse
    tg = targets if targets is not None else torch.zeros(T, dtype=torch.long, device=dev)
    a, b, c = ref.token_logprobs(logits, tg, temperature)
    if lp is not None:
        lp.copy_(a)
    if ent is not None:
        ent.copy_(b)
    if lse is not None:
        lse.copy_(c)
    if write_grad:
        z = logits.float() * inv_t
        p = torch.softmax(z, -1)
        g = -p
        if targets is not None:
            g.scatter_add_(1, targets.long().unsqueeze(1), torch.ones(T, 1, device=dev))
        logits.copy_((g * (coef.float() * inv_t).unsqueeze(1)).to(logits.dtype))
    return lp, ent, lse


def sumsq(t: torch.Tensor, out: torch.Tensor):
    """out[0] += sum(t^2) (fp32)."""
    if t.is_cuda:
        native().sumsq_accumulate(t, out)
    else:
        out += t.float().pow(2).sum()
    return out


def adamw_step(p, g, m, v, *, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, step=1,
               grad_scale=1.0, master=None, sumsq_buf=None, max_norm=0.0, seed=0):
    """Fused AdamW on flat buffers. Without ``master`` the bf16 write is
    stochastically rounded. ``sumsq_buf`` + ``max_norm`` apply global-norm
    clipping with the norm read on the device."""
    if p.is_cuda:
        native().adamw_step(p, master, g, m, v, float(lr), float(b1), float(b2), float(eps),
                            float(wd), int(step), float(grad_scale), sumsq_buf, float(max_norm),
                            int(seed) & 0x7FFFFFFF)
        return
    scale = grad_scale
    if sumsq_buf is not None and max_norm > 0:
        norm = float(sumsq_buf.sqrt()) * grad_scale
        scale *= min(1.0, max_norm / (norm + 1e-6))
    gf = g.float() * scale
    m.mul_(b1).add_(gf, alpha=1 - b1)
    v.mul_(b2).addcmul_(gf, gf, value=1 - b2)
    w = master if master is not None else p.float()
    w.mul_(1 - lr * wd)
    bc1 = 1 - b1 ** step
    bc2 = 1 - b2 ** step
    w.addcdiv_(m / bc1, (v / bc2).sqrt().add_(eps), value=-lr)
    p.copy_(w.to(p.dtype))


def adamw_step_f32(p, g, m, v, *, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, step=1,
                   grad_scale=1.0, sumsq_buf=None, max_norm=0.0):
    """AdamW for fp32 parameter buffers (tiny fp32 CPU/gloo models only)."""
    scale = grad_scale
    if sumsq_buf is not None and max_norm > 0:
        norm = float(sumsq_buf.sqrt()) * grad_scale
        scale *= min(1.0, max_norm / (norm + 1e-6))
    gf = g.float() * scale
    m.mul_(b1).add_(gf, alpha=1 - b1)
    v.mul_(b2).addcmul_(gf, gf, value=1 - b2)
    p.mul_(1 - lr * wd)
    p.addcdiv_(m / (1 - b1 ** step), (v / (1 - b2 ** step)).sqrt().add_(eps), value=-lr)
