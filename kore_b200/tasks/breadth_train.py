"""Breadth families, part 2: training-side operators.

* optimizer steps over flat parameter shards (fp32 state, parameter /
  gradient in the task dtype): AdamW (plain, AMSGrad, no decay), Adam-max,
  NAdam, RAdam, AdaGrad, AdaDelta, RMSprop (plain, centred, momentum,
  centred + momentum), SGD (momentum, Nesterov, dampening), LAMB, LARS,
  NovoGrad, Rprop, Lion, Muon's Newton-Schulz orthogonalisation (3 and 5
  steps), EMA of weights, gradient accumulation / scaling, gradient
  centring, global L2 norm, adaptive gradient clipping; each returns the
  concatenation of the updated tensors;
* loss gradients with respect to the logits: cross-entropy with label
  smoothing / z-loss / soft-capping, focal, poly-1, binary cross-entropy,
  KL / reverse-KL / Jensen-Shannon / temperature distillation, Huber, smooth
  L1, cosine-embedding.

Each operator is a module-level PyTorch definition; the fp32 oracle runs it
on fp32 copies of the inputs, the vendor baseline runs it in the task dtype,
and the seed calls it (a correct, slow starting point).
Reference parity: the training-op breadth engine of the reference
(kore/tasks/breadth/train_ops, task dirs ``genb_tr_*``), written from the
optimizer and loss definitions.
"""
from __future__ import annotations

import math
from typing import Callable, List

import torch
import torch.nn.functional as F

from .spec import OpSpec, _gen, _randn

DTYPES = ("bf16", "fp16", "fp32")
_OPT_SHAPE = {"minimal": {"N": 4096}, "primary": {"N": 64 * 1024 * 1024}, "validation": [{"N": 1000003}]}
_MAT_SHAPE = {"minimal": {"M": 64, "N": 64}, "primary": {"M": 4096, "N": 4096}, "validation": [{"M": 1024, "N": 512}]}
_LOSS_SHAPE = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 32000},
               "validation": [{"M": 333, "N": 50257}]}


def _fp32_of(f):
    return lambda *x: f(*(t.float() if t.is_floating_point() else t for t in x))


def _seed_for(entry: str, args: str, fn: Callable) -> str:
    return (f"from kore_b200.tasks.breadth_train import {fn.__name__} as _ref\n\n\n"
            f"def {entry}({args}):\n    return _ref({args})\n")


# ----------------------------------------------------------------------------- inputs
def mk_opt(d, s, dev, dt):
    n = d["N"]
    p = _randn((n,), s, dev, dt)
    g = _randn((n,), s + 1, dev, dt, 0.01)
    m = _randn((n,), s + 2, dev, torch.float32, 0.001)
    v = _randn((n,), s + 3, dev, torch.float32, 0.001).abs() + 1e-6
    return p, g, m, v


def mk_mat(d, s, dev, dt):
    return (_randn((d["M"], d["N"]), s, dev, dt, 0.1),)


def mk_logits_target(d, s, dev, dt):
    z = _randn((d["M"], d["N"]), s, dev, dt, 2.0)
    t = torch.randint(0, d["N"], (d["M"],), generator=_gen(s + 1, dev), device=dev)
    return z, t


def mk_logits_pair(d, s, dev, dt):
    return _randn((d["M"], d["N"]), s, dev, dt, 2.0), _randn((d["M"], d["N"]), s + 1, dev, dt, 2.0)


def mk_pred_target(d, s, dev, dt):
    return _randn((d["M"], d["N"]), s, dev, dt, 2.0), _randn((d["M"], d["N"]), s + 1, dev, dt, 2.0)


def mk_bce(d, s, dev, dt):
    z = _randn((d["M"], d["N"]), s, dev, dt, 2.0)
    y = (torch.rand((d["M"], d["N"]), generator=_gen(s + 1, dev), device=dev) < 0.3).to(dt)
    return z, y


# ----------------------------------------------------------------------------- optimizers
_LR, _B1, _B2, _EPS, _WD, _STEP = 1e-3, 0.9, 0.999, 1e-8, 0.01, 10


def opt_adamw(p, g, m, v):
    g = g.float()
    m2 = _B1 * m + (1 - _B1) * g
    v2 = _B2 * v + (1 - _B2) * g * g
    upd = (m2 / (1 - _B1 ** _STEP)) / ((v2 / (1 - _B2 ** _STEP)).sqrt() + _EPS)
    return torch.cat([p.float() * (1 - _LR * _WD) - _LR * upd, m2, v2])


def opt_adamw_nodecay(p, g, m, v):
    g = g.float()
    m2 = _B1 * m + (1 - _B1) * g
    v2 = _B2 * v + (1 - _B2) * g * g
    return torch.cat([p.float() - _LR * (m2 / (1 - _B1 ** _STEP)) / ((v2 / (1 - _B2 ** _STEP)).sqrt() + _EPS), m2, v2])


def opt_adamw_amsgrad(p, g, m, v):
    """``v`` holds the running max of the second moment (v_hat)."""
    g = g.float()
    m2 = _B1 * m + (1 - _B1) * g
    v2 = _B2 * v + (1 - _B2) * g * g
    vmax = torch.maximum(v, v2)
    upd = (m2 / (1 - _B1 ** _STEP)) / ((vmax / (1 - _B2 ** _STEP)).sqrt() + _EPS)
    return torch.cat([p.float() * (1 - _LR * _WD) - _LR * upd, m2, vmax])


def opt_adamax(p, g, m, v):
    g = g.float()
    m2 = _B1 * m + (1 - _B1) * g
    u = torch.maximum(_B2 * v, g.abs() + _EPS)
    return torch.cat([p.float() - (_LR / (1 - _B1 ** _STEP)) * m2 / u, m2, u])


def opt_nadam(p, g, m, v, psi=0.004):
    g = g.float()
    mu_t = _B1 * (1 - 0.5 * 0.96 ** (_STEP * psi))
    mu_n = _B1 * (1 - 0.5 * 0.96 ** ((_STEP + 1) * psi))
    prod = 1.0
    for i in range(1, _STEP + 1):
        prod *= _B1 * (1 - 0.5 * 0.96 ** (i * psi))
    m2 = _B1 * m + (1 - _B1) * g
    v2 = _B2 * v + (1 - _B2) * g * g
    vh = v2 / (1 - _B2 ** _STEP)
    upd = (mu_n * m2 / (1 - prod * mu_n) + (1 - mu_t) * g / (1 - prod)) / (vh.sqrt() + _EPS)
    return torch.cat([p.float() - _LR * upd, m2, v2])


def opt_radam(p, g, m, v):
    g = g.float()
    m2 = _B1 * m + (1 - _B1) * g
    v2 = _B2 * v + (1 - _B2) * g * g
    mh = m2 / (1 - _B1 ** _STEP)
    rho_inf = 2 / (1 - _B2) - 1
    rho = rho_inf - 2 * _STEP * _B2 ** _STEP / (1 - _B2 ** _STEP)
    if rho > 5:
        r = math.sqrt((rho - 4) * (rho - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho))
        upd = r * mh / ((v2 / (1 - _B2 ** _STEP)).sqrt() + _EPS)
    else:
        upd = mh
    return torch.cat([p.float() - _LR * upd, m2, v2])


def opt_adagrad(p, g, m, v):
    g = g.float()
    v2 = v + g * g
    return torch.cat([p.float() - 1e-2 * g / (v2.sqrt() + 1e-10), v2])


def opt_adadelta(p, g, m, v, rho=0.9, eps=1e-6):
    """``v``: running E[g^2]; ``m``: running E[dx^2] (squared, non-negative)."""
    g = g.float()
    acc_dx = m * m
    v2 = rho * v + (1 - rho) * g * g
    dx = (acc_dx + eps).sqrt() / (v2 + eps).sqrt() * g
    acc2 = rho * acc_dx + (1 - rho) * dx * dx
    return torch.cat([p.float() - dx, v2, acc2])


def opt_rmsprop(p, g, m, v, alpha=0.99, eps=1e-8, lr=1e-2):
    g = g.float()
    v2 = alpha * v + (1 - alpha) * g * g
    return torch.cat([p.float() - lr * g / (v2.sqrt() + eps), v2])


def opt_rmsprop_centered(p, g, m, v, alpha=0.99, eps=1e-8, lr=1e-2):
    g = g.float()
    v2 = alpha * v + (1 - alpha) * g * g
    ga = alpha * m + (1 - alpha) * g
    return torch.cat([p.float() - lr * g / ((v2 - ga * ga).clamp_min(0).sqrt() + eps), v2, ga])


def opt_rmsprop_momentum(p, g, m, v, alpha=0.99, eps=1e-8, lr=1e-2, mu=0.9):
    g = g.float()
    v2 = alpha * v + (1 - alpha) * g * g
    buf = mu * m + g / (v2.sqrt() + eps)
    return torch.cat([p.float() - lr * buf, v2, buf])


def opt_rmsprop_centered_momentum(p, g, m, v, alpha=0.99, eps=1e-8, lr=1e-2, mu=0.9):
    g = g.float()
    v2 = alpha * v + (1 - alpha) * g * g
    ga = alpha * (m * 0.5) + (1 - alpha) * g
    buf = mu * m + g / ((v2 - ga * ga).clamp_min(0).sqrt() + eps)
    return torch.cat([p.float() - lr * buf, v2, ga, buf])


def opt_sgd_momentum(p, g, m, v, lr=1e-2, mu=0.9):
    buf = mu * m + g.float()
    return torch.cat([p.float() - lr * buf, buf])


def opt_sgd_nesterov(p, g, m, v, lr=1e-2, mu=0.9):
    g = g.float()
    buf = mu * m + g
    return torch.cat([p.float() - lr * (g + mu * buf), buf])


def opt_sgd_dampening(p, g, m, v, lr=1e-2, mu=0.9, damp=0.1, wd=1e-4):
    g = g.float() + wd * p.float()
    buf = mu * m + (1 - damp) * g
    return torch.cat([p.float() - lr * buf, buf])


def opt_lamb(p, g, m, v):
    g = g.float()
    pf = p.float()
    m2 = _B1 * m + (1 - _B1) * g
    v2 = _B2 * v + (1 - _B2) * g * g
    r = (m2 / (1 - _B1 ** _STEP)) / ((v2 / (1 - _B2 ** _STEP)).sqrt() + 1e-6) + _WD * pf
    wn, rn = pf.norm(), r.norm()
    trust = torch.where((wn > 0) & (rn > 0), wn / rn, torch.ones_like(wn))
    return torch.cat([pf - _LR * trust * r, m2, v2])


def opt_lars(p, g, m, v, lr=1e-2, mu=0.9, wd=1e-4, eta=1e-3):
    g = g.float()
    pf = p.float()
    wn, gn = pf.norm(), g.norm()
    local = torch.where((wn > 0) & (gn > 0), eta * wn / (gn + wd * wn), torch.ones_like(wn))
    buf = mu * m + local * lr * (g + wd * pf)
    return torch.cat([pf - buf, buf])


def opt_novograd(p, g, m, v, lr=1e-3, b1=0.95, b2=0.98, wd=1e-3, eps=1e-8):
    """Layer-wise second moment: ``v[0]`` holds the running squared norm."""
    g = g.float()
    pf = p.float()
    vn = b2 * v[0] + (1 - b2) * (g * g).sum()
    m2 = b1 * m + (g / (vn.sqrt() + eps) + wd * pf)
    return torch.cat([pf - lr * m2, m2, vn.reshape(1)])


def opt_rprop(p, g, m, v, eta_plus=1.2, eta_minus=0.5, smin=1e-6, smax=50.0):
    """``m``: previous gradient; ``v``: per-element step sizes."""
    g = g.float()
    sgn = torch.sign(g * m)
    step = torch.where(sgn > 0, (v * eta_plus).clamp(max=smax), torch.where(sgn < 0, (v * eta_minus).clamp(min=smin), v))
    g2 = torch.where(sgn < 0, torch.zeros_like(g), g)
    return torch.cat([p.float() - torch.sign(g2) * step, g2, step])


def opt_lion(p, g, m, v, lr=1e-4, b1=0.9, b2=0.99, wd=0.01):
    g = g.float()
    c = torch.sign(b1 * m + (1 - b1) * g)
    return torch.cat([p.float() * (1 - lr * wd) - lr * c, b2 * m + (1 - b2) * g])


def opt_ema_update(p, g, m, v, decay=0.999):
    """EMA of weights: ``m`` is the shadow copy, ``p`` the live weights."""
    return decay * m + (1 - decay) * p.float()


def opt_grad_accum_scale(p, g, m, v, scale=0.125):
    return m + scale * g.float()


def opt_grad_zero_center(p, g, m, v):
    gf = g.float()
    return gf - gf.mean()


def opt_global_l2_norm(p, g, m, v):
    return g.float().pow(2).sum().sqrt().reshape(1)


def opt_agc(p, g, m, v, clip=0.01, eps=1e-3):
    """Adaptive gradient clipping on one unit: ||g|| <= clip * max(||p||, eps)."""
    gf, pf = g.float(), p.float()
    mx = clip * torch.clamp(pf.norm(), min=eps)
    gn = gf.norm()
    return torch.where(gn > mx, gf * (mx / (gn + 1e-6)), gf)


def muon_ns3(x):
    return _newton_schulz(x, 3)


def muon_ns5(x):
    return _newton_schulz(x, 5)


def _newton_schulz(x, steps):
    """Approximate orthogonalisation with the quintic iteration used by Muon
    (coefficients 3.4445, -4.7750, 2.0315)."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = x.float()
    X = X / (X.norm() + 1e-7)
    t = X.shape[0] > X.shape[1]
    if t:
        X = X.t()
    for _ in range(steps):
        A = X @ X.t()
        X = a * X + (b * A + c * A @ A) @ X
    return X.t() if t else X


OPTIMIZERS = [opt_adamw, opt_adamw_nodecay, opt_adamw_amsgrad, opt_adamax, opt_nadam, opt_radam, opt_adagrad,
              opt_adadelta, opt_rmsprop, opt_rmsprop_centered, opt_rmsprop_momentum, opt_rmsprop_centered_momentum,
              opt_sgd_momentum, opt_sgd_nesterov, opt_sgd_dampening, opt_lamb, opt_lars, opt_novograd, opt_rprop,
              opt_lion, opt_ema_update, opt_grad_accum_scale, opt_grad_zero_center, opt_global_l2_norm, opt_agc]


# ----------------------------------------------------------------------------- loss gradients
def _dlogits(loss: Callable, z: torch.Tensor, *rest) -> torch.Tensor:
    """d loss / d z (mean over rows) by autograd on a detached copy."""
    with torch.enable_grad():
        zz = z.detach().requires_grad_(True)
        (gz,) = torch.autograd.grad(loss(zz, *rest), zz)
    return gz


def ce_label_smoothing_bwd(z, t):
    return _dlogits(lambda a, b: F.cross_entropy(a, b, label_smoothing=0.1), z, t)


def ce_zloss_bwd(z, t):
    return _dlogits(lambda a, b: F.cross_entropy(a, b) + 1e-4 * torch.logsumexp(a, -1).pow(2).mean(), z, t)


def ce_softcap_bwd(z, t, cap=30.0):
    return _dlogits(lambda a, b: F.cross_entropy(cap * torch.tanh(a / cap), b), z, t)


def ce_focal_bwd(z, t, gamma=2.0):
    def loss(a, b):
        lp = torch.log_softmax(a, -1).gather(-1, b[:, None]).squeeze(-1)
        return (-(1 - lp.exp()).pow(gamma) * lp).mean()
    return _dlogits(loss, z, t)


def ce_poly1_bwd(z, t, eps=1.0):
    def loss(a, b):
        pt = torch.softmax(a, -1).gather(-1, b[:, None]).squeeze(-1)
        return (F.cross_entropy(a, b, reduction="none") + eps * (1 - pt)).mean()
    return _dlogits(loss, z, t)


def ce_bwd(z, t):
    return _dlogits(lambda a, b: F.cross_entropy(a, b), z, t)


def bce_logits_bwd(z, y):
    return _dlogits(lambda a, b: F.binary_cross_entropy_with_logits(a, b), z, y)


def kl_distill_bwd(z, zt):
    return _dlogits(lambda a, b: F.kl_div(torch.log_softmax(a, -1), torch.log_softmax(b, -1), log_target=True,
                                          reduction="batchmean"), z, zt)


def reverse_kl_distill_bwd(z, zt):
    return _dlogits(lambda a, b: F.kl_div(torch.log_softmax(b, -1), torch.log_softmax(a, -1), log_target=True,
                                          reduction="batchmean"), z, zt)


def js_distill_bwd(z, zt):
    def loss(a, b):
        p, q = torch.softmax(a, -1), torch.softmax(b, -1)
        mlog = (0.5 * (p + q)).clamp_min(1e-30).log()
        return 0.5 * (F.kl_div(mlog, p, reduction="batchmean") + F.kl_div(mlog, q, reduction="batchmean"))
    return _dlogits(loss, z, zt)


def temp_distill_bwd(z, zt, T=2.0):
    return _dlogits(lambda a, b: T * T * F.kl_div(torch.log_softmax(a / T, -1), torch.log_softmax(b / T, -1),
                                                  log_target=True, reduction="batchmean"), z, zt)


def huber_bwd(x, y):
    return _dlogits(lambda a, b: F.huber_loss(a, b, delta=1.0), x, y)


def smooth_l1_bwd(x, y):
    return _dlogits(lambda a, b: F.smooth_l1_loss(a, b, beta=0.5), x, y)


def cosine_embed_bwd(x, y):
    return _dlogits(lambda a, b: (1 - F.cosine_similarity(a, b, dim=-1)).mean(), x, y)


LOSSES = [(ce_bwd, mk_logits_target, "z, t"), (ce_label_smoothing_bwd, mk_logits_target, "z, t"),
          (ce_zloss_bwd, mk_logits_target, "z, t"), (ce_softcap_bwd, mk_logits_target, "z, t"),
          (ce_focal_bwd, mk_logits_target, "z, t"), (ce_poly1_bwd, mk_logits_target, "z, t"),
          (bce_logits_bwd, mk_bce, "z, y"), (kl_distill_bwd, mk_logits_pair, "z, zt"),
          (reverse_kl_distill_bwd, mk_logits_pair, "z, zt"), (js_distill_bwd, mk_logits_pair, "z, zt"),
          (temp_distill_bwd, mk_logits_pair, "z, zt"), (huber_bwd, mk_pred_target, "x, y"),
          (smooth_l1_bwd, mk_pred_target, "x, y"), (cosine_embed_bwd, mk_pred_target, "x, y")]


def build() -> List[OpSpec]:
    out: List[OpSpec] = []
    for dt in DTYPES:
        for fn in OPTIMIZERS:
            nm = fn.__name__[4:]
            out.append(OpSpec(f"genb_tr_{nm}_{dt}", "optimizer", "step", mk_opt, _fp32_of(fn), fn,
                              _seed_for("step", "p, g, m, v", fn), _OPT_SHAPE, "train", dt))
        for fn in (muon_ns3, muon_ns5):
            out.append(OpSpec(f"genb_tr_{fn.__name__}_{dt}", "newton_schulz", "orthogonalize", mk_mat, _fp32_of(fn), fn,
                              _seed_for("orthogonalize", "x", fn), _MAT_SHAPE, "train", dt))
        for fn, mk, args in LOSSES:
            out.append(OpSpec(f"genb_tr_{fn.__name__}_{dt}", "loss_bwd", "loss_grad", mk, _fp32_of(fn), fn,
                              _seed_for("loss_grad", args, fn), _LOSS_SHAPE, "train", dt))
    return out
