"""Breadth families, part 3: convolutions, state-space / linear-recurrence
models, sampling, normalisations and reductions.

* conv: 1-D (kernel 3 / 5, stride 2, dilation 2), 2-D (1x1, 3x3, 3x3 stride
  2, 5x5, dilated, grouped, depthwise), transposed 2-D, 3-D, pooling
  (max / avg with strides, adaptive average) and interpolation (nearest,
  bilinear);
* ssm: Mamba selective scan, Mamba-2 chunked state-space dual, gated linear
  attention, RetNet retention, RWKV-style time mixing, S4-style
  discretisation, causal linear attention, exponential moving average;
* sampling: top-k + top-p, typical-p, frequency / presence penalties, logit
  soft-capping, Gumbel-max with a fixed noise tensor, beam-score update,
  per-row entropy;
* norm: group norm, instance norm, batch norm (training statistics),
  LayerNorm / RMSNorm backward, L2 row normalisation, scale norm, per-head
  q/k RMSNorm, DeepNorm residual;
* reductions: variance / std, log-sum-exp, arg-max, column means, p-norms,
  cumulative max, segment sums, softmax cross-row statistics.

Each operator is a module-level PyTorch definition (fp32 oracle on fp32
copies, vendor baseline in the task dtype, seed calling it).
Reference parity: the breadth engines of the reference (task dirs
``genb_cv_*``, ``genb_ssm_*``, ``genb_smp_*``, ``genb_norm_*``, ``genb_red_*``),
written from the operator definitions.
"""
from __future__ import annotations

import math
from typing import Callable, List

import torch
import torch.nn.functional as F

from .spec import OpSpec, _gen, _randn


def _fp32_of(f):
    return lambda *x: f(*(t.float() if t.is_floating_point() else t for t in x))


def _seed_for(entry: str, args: str, fn: Callable) -> str:
    return (f"from kore_b200.tasks.breadth_ext import {fn.__name__} as _ref\n\n\n"
            f"def {entry}({args}):\n    return _ref({args})\n")


# ============================================================================= conv
def mk_img(d, s, dev, dt):
    x = _randn((d["B"], d["C"], d["H"], d["H"]), s, dev, dt)
    w = _randn((d["C"], d["C"], 3, 3), s + 1, dev, dt, 1.0 / math.sqrt(9 * d["C"]))
    return x, w


def mk_seq1d(d, s, dev, dt):
    x = _randn((d["B"], d["C"], d["L"]), s, dev, dt)
    w = _randn((d["C"], d["C"], 5), s + 1, dev, dt, 1.0 / math.sqrt(5 * d["C"]))
    return x, w


def mk_vol(d, s, dev, dt):
    x = _randn((d["B"], d["C"], 16, d["H"], d["H"]), s, dev, dt)
    w = _randn((d["C"], d["C"], 3, 3, 3), s + 1, dev, dt, 1.0 / math.sqrt(27 * d["C"]))
    return x, w


def conv1d_k3(x, w):
    return F.conv1d(x, w[..., 1:4], padding=1)


def conv1d_k5(x, w):
    return F.conv1d(x, w, padding=2)


def conv1d_k5_stride2(x, w):
    return F.conv1d(x, w, stride=2, padding=2)


def conv1d_k3_dilation2(x, w):
    return F.conv1d(x, w[..., 1:4], padding=2, dilation=2)


def conv2d_1x1(x, w):
    return F.conv2d(x, w[..., 1:2, 1:2])


def conv2d_3x3_stride2(x, w):
    return F.conv2d(x, w, stride=2, padding=1)


def conv2d_3x3_dilation2(x, w):
    return F.conv2d(x, w, padding=2, dilation=2)


def conv2d_3x3_groups4(x, w):
    C = x.shape[1]
    return F.conv2d(x, w[: C, : C // 4], padding=1, groups=4)


def conv2d_depthwise3x3(x, w):
    C = x.shape[1]
    return F.conv2d(x, w[:, :1], padding=1, groups=C)


def conv2d_5x5(x, w):
    return F.conv2d(x, F.pad(w, (1, 1, 1, 1)), padding=2)


def conv_transpose2d_3x3_stride2(x, w):
    return F.conv_transpose2d(x, w, stride=2, padding=1, output_padding=1)


def conv3d_3x3x3(x, w):
    return F.conv3d(x, w, padding=1)


def maxpool2d_3x3_stride2(x, w):
    return F.max_pool2d(x, 3, stride=2, padding=1)


def avgpool2d_3x3_stride1(x, w):
    return F.avg_pool2d(x, 3, stride=1, padding=1)


def adaptive_avgpool_7x7(x, w):
    return F.adaptive_avg_pool2d(x, 7)


def upsample_nearest2x(x, w):
    return F.interpolate(x, scale_factor=2, mode="nearest")


def upsample_bilinear2x(x, w):
    return F.interpolate(x, scale_factor=2, mode="bilinear", align_corners=False)


CONV2D = [conv2d_1x1, conv2d_3x3_stride2, conv2d_3x3_dilation2, conv2d_3x3_groups4, conv2d_depthwise3x3,
          conv2d_5x5, conv_transpose2d_3x3_stride2, maxpool2d_3x3_stride2, avgpool2d_3x3_stride1,
          adaptive_avgpool_7x7, upsample_nearest2x, upsample_bilinear2x]
CONV1D = [conv1d_k3, conv1d_k5, conv1d_k5_stride2, conv1d_k3_dilation2]


# ============================================================================= ssm
def mk_selective(d, s, dev, dt):
    B, L, D, N = d["B"], d["L"], d["D"], d["N"]
    x = _randn((B, L, D), s, dev, dt)
    delta = (F.softplus(_randn((B, L, D), s + 1, dev, torch.float32) - 2)).to(dt)
    A = (-torch.exp(_randn((D, N), s + 2, dev, torch.float32, 0.5))).to(dt)
    Bm = _randn((B, L, N), s + 3, dev, dt)
    Cm = _randn((B, L, N), s + 4, dev, dt)
    return x, delta, A, Bm, Cm


def selective_scan(x, delta, A, Bm, Cm):
    """h_t = exp(delta_t A) h_{t-1} + delta_t B_t x_t,  y_t = C_t . h_t."""
    B, L, D = x.shape
    h = torch.zeros(B, D, A.shape[1], dtype=torch.float32, device=x.device)
    ys = []
    for t in range(L):
        dA = torch.exp(delta[:, t, :, None].float() * A.float())
        h = dA * h + (delta[:, t, :, None] * x[:, t, :, None]).float() * Bm[:, t, None, :].float()
        ys.append((h * Cm[:, t, None, :].float()).sum(-1))
    return torch.stack(ys, 1)


def mk_gla(d, s, dev, dt):
    B, L, H, K = d["B"], d["L"], d["H"], d["K"]
    q = _randn((B, H, L, K), s, dev, dt, K ** -0.5)
    k = _randn((B, H, L, K), s + 1, dev, dt, K ** -0.5)
    v = _randn((B, H, L, K), s + 2, dev, dt)
    g = torch.sigmoid(_randn((B, H, L, K), s + 3, dev, torch.float32) + 3).to(dt)
    return q, k, v, g


def gated_linear_attention(q, k, v, g):
    """S_t = diag(g_t) S_{t-1} + k_t v_t^T;  o_t = q_t^T S_t."""
    B, H, L, K = q.shape
    S = torch.zeros(B, H, K, v.shape[-1], device=q.device)
    out = []
    for t in range(L):
        S = g[:, :, t, :, None].float() * S + k[:, :, t, :, None].float() * v[:, :, t, None, :].float()
        out.append(torch.einsum("bhk,bhkv->bhv", q[:, :, t].float(), S))
    return torch.stack(out, 2)


def retention(q, k, v, g):
    """RetNet retention with a per-head scalar decay gamma_h in (0.9, 1)."""
    B, H, L, K = q.shape
    gamma = 1 - torch.exp2(-5 - torch.arange(H, device=q.device, dtype=torch.float32) * 0.25)
    n = torch.arange(L, device=q.device, dtype=torch.float32)
    Dm = torch.where(n[:, None] >= n[None, :], gamma[:, None, None] ** (n[:, None] - n[None, :]), torch.zeros(()))
    att = torch.einsum("bhik,bhjk->bhij", q.float(), k.float()) * Dm[None]
    return att @ v.float()


def causal_linear_attention(q, k, v, g):
    qf, kf = F.elu(q.float()) + 1, F.elu(k.float()) + 1
    att = torch.einsum("bhik,bhjk->bhij", qf, kf).tril()
    return (att @ v.float()) / (att.sum(-1, keepdim=True) + 1e-6)


def rwkv_time_mix(q, k, v, g):
    """WKV with per-channel decay w = g (in (0,1)) and bonus u = 0.5:
    o_t = (sum_{i<t} w^{t-1-i} e^{k_i} v_i + e^{u + k_t} v_t) / (same sums of e^k)."""
    B, H, L, K = k.shape
    kf, vf, w = k.float(), v.float(), g[:, :, 0, :].float()
    num = torch.zeros(B, H, K, device=k.device)
    den = torch.zeros(B, H, K, device=k.device)
    out = []
    for t in range(L):
        ek = torch.exp(kf[:, :, t])
        bonus = torch.exp(0.5 + kf[:, :, t])
        out.append((num + bonus * vf[:, :, t]) / (den + bonus))
        num = w * num + ek * vf[:, :, t]
        den = w * den + ek
    return torch.stack(out, 2)


def ssd_chunked(q, k, v, g):
    """Mamba-2 state-space dual with scalar decay per head and step (the
    first channel of g), evaluated in chunks of 64 (quadratic inside a chunk,
    a carried state across chunks)."""
    B, H, L, K = q.shape
    a = g[..., 0].float().clamp_min(1e-4).log()                      # log decay [B,H,L]
    C = 64
    S = torch.zeros(B, H, K, v.shape[-1], device=q.device)
    outs = []
    for c0 in range(0, L, C):
        qa, ka, va, aa = (t[:, :, c0:c0 + C].float() for t in (q, k, v, a[..., None]))
        aa = aa[..., 0]
        cum = aa.cumsum(-1)
        seg = cum[..., :, None] - cum[..., None, :]
        Lm = torch.where(seg.new_ones(seg.shape[-1], seg.shape[-1]).tril().bool(), seg.exp(), torch.zeros(()))
        y = torch.einsum("bhik,bhjk->bhij", qa, ka) * Lm
        y = y @ va + torch.einsum("bhik,bhkv->bhiv", qa * cum.exp()[..., None], S)
        outs.append(y)
        S = S * cum[..., -1:, None].exp() + torch.einsum("bhjk,bhjv->bhkv", ka * (cum[..., -1:] - cum).exp()[..., None], va)
    return torch.cat(outs, 2)


def mk_ema(d, s, dev, dt):
    return _randn((d["B"], d["L"], d["D"]), s, dev, dt), torch.sigmoid(_randn((d["D"],), s + 1, dev, torch.float32)).to(dt)


def ema_scan(x, a):
    y, h = [], torch.zeros_like(x[:, 0].float())
    for t in range(x.shape[1]):
        h = a.float() * h + (1 - a.float()) * x[:, t].float()
        y.append(h)
    return torch.stack(y, 1)


def mk_s4(d, s, dev, dt):
    A = -torch.exp(_randn((d["D"], d["N"]), s, dev, torch.float32, 0.5)).to(dt)
    delta = F.softplus(_randn((d["D"],), s + 1, dev, torch.float32)).to(dt)
    return A, delta


def s4_discretize(A, delta):
    """Zero-order hold: (exp(delta A), (exp(delta A) - 1) / A)."""
    dA = torch.exp(delta[:, None] * A)
    return torch.cat([dA, (dA - 1) / A], -1)


GLA_FAMILY = [gated_linear_attention, retention, causal_linear_attention, rwkv_time_mix, ssd_chunked]


# ============================================================================= sampling
def mk_logits(d, s, dev, dt):
    return (_randn((d["M"], d["V"]), s, dev, dt, 3.0),)


def mk_logits_counts(d, s, dev, dt):
    z = _randn((d["M"], d["V"]), s, dev, dt, 3.0)
    c = torch.randint(0, 4, (d["M"], d["V"]), generator=_gen(s + 1, dev), device=dev)
    c = c * (torch.rand((d["M"], d["V"]), generator=_gen(s + 2, dev), device=dev) < 0.01)
    return z, c


def mk_logits_noise(d, s, dev, dt):
    z = _randn((d["M"], d["V"]), s, dev, dt, 3.0)
    u = torch.rand((d["M"], d["V"]), generator=_gen(s + 3, dev), device=dev).clamp(1e-6, 1 - 1e-6)
    return z, u


def topk_topp_probs(z, k=50, p=0.9):
    zf = z.float()
    kth = zf.topk(k, -1).values[..., -1:]
    zf = zf.masked_fill(zf < kth, float("-inf"))
    pr = torch.softmax(zf, -1)
    sp, idx = pr.sort(-1, descending=True)
    keep = (sp.cumsum(-1) - sp) < p
    mask = torch.zeros_like(keep).scatter(-1, idx, keep)
    pr = pr * mask
    return pr / pr.sum(-1, keepdim=True)


def typical_p_probs(z, mass=0.95):
    lp = torch.log_softmax(z.float(), -1)
    pr = lp.exp()
    ent = -(pr * lp).sum(-1, keepdim=True)
    dev = (-lp - ent).abs()
    order = dev.argsort(-1)
    sp = pr.gather(-1, order)
    keep = (sp.cumsum(-1) - sp) < mass
    mask = torch.zeros_like(keep).scatter(-1, order, keep)
    q = pr * mask
    return q / q.sum(-1, keepdim=True)


def freq_presence_penalty(z, c, fp=0.5, pp=0.3):
    return z.float() - fp * c.float() - pp * (c > 0).float()


def logit_softcap(z, cap=30.0):
    return cap * torch.tanh(z.float() / cap)


def gumbel_argmax_onehot(z, u):
    g = -torch.log(-torch.log(u.float()))
    i = (z.float() + g).argmax(-1)
    return F.one_hot(i, z.shape[-1]).float()


def beam_score_update(z, c):
    """Running beam scores (the count tensor's row sums as previous scores) plus
    log-probabilities: the top 8 candidates per row, values then indices."""
    prev = c.float().sum(-1, keepdim=True) * -0.1
    s = prev + torch.log_softmax(z.float(), -1)
    v, i = s.topk(8, -1)
    return torch.cat([v, i.float()], -1)


def row_entropy(z):
    lp = torch.log_softmax(z.float(), -1)
    return -(lp.exp() * lp).sum(-1)


SAMPLING = [(topk_topp_probs, mk_logits, "z"), (typical_p_probs, mk_logits, "z"),
            (freq_presence_penalty, mk_logits_counts, "z, c"), (logit_softcap, mk_logits, "z"),
            (gumbel_argmax_onehot, mk_logits_noise, "z, u"), (beam_score_update, mk_logits_counts, "z, c"),
            (row_entropy, mk_logits, "z")]


# ============================================================================= norms
def mk_act4d(d, s, dev, dt):
    x = _randn((d["B"], d["C"], d["H"], d["H"]), s, dev, dt)
    w = (1 + 0.1 * _randn((d["C"],), s + 1, dev, torch.float32)).to(dt)
    b = (0.1 * _randn((d["C"],), s + 2, dev, torch.float32)).to(dt)
    return x, w, b


def group_norm32(x, w, b):
    return F.group_norm(x, 32, w, b, 1e-5)


def instance_norm(x, w, b):
    return F.instance_norm(x, weight=w, bias=b, eps=1e-5)


def batch_norm_train(x, w, b):
    return F.batch_norm(x, None, None, w, b, training=True, eps=1e-5)


def mk_rows_grad(d, s, dev, dt):
    x = _randn((d["M"], d["N"]), s, dev, dt)
    w = (1 + 0.1 * _randn((d["N"],), s + 1, dev, torch.float32)).to(dt)
    g = _randn((d["M"], d["N"]), s + 2, dev, dt)
    return x, w, g


def layernorm_bwd(x, w, g):
    with torch.enable_grad():
        xx, ww = x.detach().requires_grad_(True), w.detach().requires_grad_(True)
        y = F.layer_norm(xx, xx.shape[-1:], ww, None, 1e-5)
        dx, dw = torch.autograd.grad(y, (xx, ww), g)
    return torch.cat([dx.reshape(-1), dw.reshape(-1)])


def rmsnorm_bwd(x, w, g):
    with torch.enable_grad():
        xx, ww = x.detach().requires_grad_(True), w.detach().requires_grad_(True)
        y = xx * torch.rsqrt(xx.pow(2).mean(-1, keepdim=True) + 1e-6) * ww
        dx, dw = torch.autograd.grad(y, (xx, ww), g)
    return torch.cat([dx.reshape(-1), dw.reshape(-1)])


def l2_normalize(x, w, g):
    return F.normalize(x.float(), dim=-1)


def scale_norm(x, w, g):
    return x * (w.float().mean() / x.float().norm(dim=-1, keepdim=True).clamp_min(1e-5))


def deepnorm_residual(x, w, g, alpha=2.0):
    """LayerNorm(alpha * x + f(x)) with the sublayer output given as ``g``."""
    return F.layer_norm(alpha * x + g, x.shape[-1:], w, None, 1e-5)


def mk_heads(d, s, dev, dt):
    x = _randn((d["M"], d["H"] * 128), s, dev, dt)
    w = (1 + 0.1 * _randn((128,), s + 1, dev, torch.float32)).to(dt)
    return x, w


def qk_head_rmsnorm(x, w):
    xs = x.float().view(x.shape[0], -1, 128)
    return (xs * torch.rsqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).view(x.shape)


NORM4D = [group_norm32, instance_norm, batch_norm_train]
NORMROW = [layernorm_bwd, rmsnorm_bwd, l2_normalize, scale_norm, deepnorm_residual]


# ============================================================================= reductions
def mk_rows(d, s, dev, dt):
    return (_randn((d["M"], d["N"]), s, dev, dt),)


def mk_rows_segments(d, s, dev, dt):
    x = _randn((d["M"], d["N"]), s, dev, dt)
    seg = torch.randint(0, 64, (d["M"],), generator=_gen(s + 1, dev), device=dev).sort().values
    return x, seg


def row_var(x):
    return x.float().var(-1)


def row_std(x):
    return x.float().std(-1)


def row_logsumexp(x):
    return torch.logsumexp(x.float(), -1)


def row_argmax(x):
    return x.float().argmax(-1).float()


def col_mean(x):
    return x.float().mean(0)


def col_max(x):
    return x.float().amax(0)


def row_p3_norm(x):
    return x.float().abs().pow(3).sum(-1).pow(1.0 / 3)


def row_cummax(x):
    return x.float().cummax(-1).values


def row_cumsum_reverse(x):
    return x.float().flip(-1).cumsum(-1).flip(-1)


def row_softmax_stats(x):
    """Per-row max and log-sum-exp (the two statistics a split softmax keeps)."""
    xf = x.float()
    return torch.stack([xf.amax(-1), torch.logsumexp(xf, -1)], -1)


def segment_sum(x, seg):
    out = torch.zeros(64, x.shape[1], device=x.device)
    return out.index_add_(0, seg, x.float())


def row_mean_abs_dev(x):
    xf = x.float()
    return (xf - xf.mean(-1, keepdim=True)).abs().mean(-1)


REDUCTIONS = [row_var, row_std, row_logsumexp, row_argmax, col_mean, col_max, row_p3_norm, row_cummax,
              row_cumsum_reverse, row_softmax_stats, row_mean_abs_dev]


# ============================================================================= assembly
def build() -> List[OpSpec]:
    out: List[OpSpec] = []
    for dt in ("bf16", "fp16"):
        for (B, C, H) in ((16, 128, 64), (4, 256, 128)):
            sh = {"minimal": {"B": 1, "C": 32, "H": 16}, "primary": {"B": B, "C": C, "H": H}, "validation": []}
            for fn in CONV2D:
                out.append(OpSpec(f"genb_cv_{fn.__name__}_c{C}h{H}_{dt}", "conv", "conv", mk_img, _fp32_of(fn), fn,
                                  _seed_for("conv", "x, w", fn), sh, "conv", dt))
            for fn in NORM4D:
                out.append(OpSpec(f"genb_norm_{fn.__name__}_c{C}h{H}_{dt}", "norm", "norm", mk_act4d, _fp32_of(fn),
                                  fn, _seed_for("norm", "x, w, b", fn), sh, "norm", dt))
        for (B, C, L) in ((8, 512, 4096), (32, 256, 1024)):
            sh = {"minimal": {"B": 1, "C": 16, "L": 64}, "primary": {"B": B, "C": C, "L": L}, "validation": []}
            for fn in CONV1D:
                out.append(OpSpec(f"genb_cv_{fn.__name__}_c{C}l{L}_{dt}", "conv", "conv", mk_seq1d, _fp32_of(fn), fn,
                                  _seed_for("conv", "x, w", fn), sh, "conv", dt))
        sh3 = {"minimal": {"B": 1, "C": 8, "H": 8}, "primary": {"B": 4, "C": 64, "H": 64}, "validation": []}
        out.append(OpSpec(f"genb_cv_conv3d_3x3x3_c64h64_{dt}", "conv", "conv", mk_vol, _fp32_of(conv3d_3x3x3),
                          conv3d_3x3x3, _seed_for("conv", "x, w", conv3d_3x3x3), sh3, "conv", dt))
        for (B, L, D, N) in ((4, 2048, 1024, 16), (1, 4096, 2048, 16)):
            sh = {"minimal": {"B": 1, "L": 32, "D": 16, "N": 4}, "primary": {"B": B, "L": L, "D": D, "N": N},
                  "validation": []}
            out.append(OpSpec(f"genb_ssm_selective_scan_b{B}l{L}d{D}_{dt}", "scan", "scan", mk_selective,
                              _fp32_of(selective_scan), selective_scan,
                              _seed_for("scan", "x, delta, A, Bm, Cm", selective_scan), sh, "ssm", dt))
        for (B, H, L) in ((4, 16, 2048), (1, 32, 4096)):
            sh = {"minimal": {"B": 1, "H": 2, "L": 128, "K": 64}, "primary": {"B": B, "H": H, "L": L, "K": 128},
                  "validation": []}
            for fn in GLA_FAMILY:
                out.append(OpSpec(f"genb_ssm_{fn.__name__}_b{B}h{H}l{L}_{dt}", "linear_attention", "mix", mk_gla,
                                  _fp32_of(fn), fn, _seed_for("mix", "q, k, v, g", fn), sh, "ssm", dt))
        shema = {"minimal": {"B": 1, "L": 64, "D": 32}, "primary": {"B": 8, "L": 4096, "D": 2048}, "validation": []}
        out.append(OpSpec(f"genb_ssm_ema_scan_{dt}", "scan", "scan", mk_ema, _fp32_of(ema_scan), ema_scan,
                          _seed_for("scan", "x, a", ema_scan), shema, "ssm", dt))
        shs4 = {"minimal": {"D": 16, "N": 8}, "primary": {"D": 8192, "N": 64}, "validation": []}
        out.append(OpSpec(f"genb_ssm_s4_discretize_{dt}", "elementwise", "discretize", mk_s4, _fp32_of(s4_discretize),
                          s4_discretize, _seed_for("discretize", "A, delta", s4_discretize), shs4, "ssm", dt))
        for V in (32000, 151936):
            sh = {"minimal": {"M": 4, "V": 1024}, "primary": {"M": 256, "V": V}, "validation": []}
            for fn, mk, args in SAMPLING:
                out.append(OpSpec(f"genb_smp_{fn.__name__}_v{V}_{dt}", "softmax", "sample", mk, _fp32_of(fn), fn,
                                  _seed_for("sample", args, fn), sh, "sample", dt))
        for (M, N) in ((8192, 4096), (4096, 8192)):
            sh = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": M, "N": N}, "validation": [{"M": 333, "N": 2048}]}
            for fn in NORMROW:
                out.append(OpSpec(f"genb_norm_{fn.__name__}_m{M}n{N}_{dt}", "norm", "norm", mk_rows_grad, _fp32_of(fn),
                                  fn, _seed_for("norm", "x, w, g", fn), sh, "norm", dt))
            for fn in REDUCTIONS:
                out.append(OpSpec(f"genb_red_{fn.__name__}_m{M}n{N}_{dt}", "reduce", "reduce", mk_rows, _fp32_of(fn),
                                  fn, _seed_for("reduce", "x", fn), sh, "reduce", dt))
            out.append(OpSpec(f"genb_red_segment_sum_m{M}n{N}_{dt}", "reduce", "reduce", mk_rows_segments,
                              _fp32_of(segment_sum), segment_sum, _seed_for("reduce", "x, seg", segment_sum), sh,
                              "reduce", dt))
        for H in (32, 40, 64):
            sh = {"minimal": {"M": 16, "H": 2}, "primary": {"M": 8192, "H": H}, "validation": []}
            out.append(OpSpec(f"genb_norm_qk_head_rmsnorm_h{H}_{dt}", "norm", "norm", mk_heads,
                              _fp32_of(qk_head_rmsnorm), qk_head_rmsnorm, _seed_for("norm", "x, w", qk_head_rmsnorm),
                              sh, "norm", dt))
    return out
