"""Metamorphic relations: identities an implementation of an operator class
must satisfy, checked without the reference.

elementwise  - equivariance under a permutation of the flattened input,
               locality (perturbing one element changes only that output),
               reshape invariance;
reduction    - (row-wise reductions / normalisations over the last axis)
               equivariance under a row permutation, row locality, and
               invariance (or equivariance, for row-shaped outputs) under a
               permutation inside the rows;
generic      - no structural identity is assumed.

Each relation is ``rel(fn, *inputs, rtol=...) -> (ok, detail)``; the
perturbations are deterministic so a failure reproduces.
Reference behaviour: kore/verify/metamorphic.py:1-205.
"""
from __future__ import annotations

from typing import Callable, List, Tuple

import torch

ELEMENTWISE = ("elementwise", "unary", "binary", "activation", "pointwise")
REDUCTION = ("reduce", "reduction", "norm", "softmax", "row")


def _close(a, b, rtol: float) -> bool:
    a, b = a.float(), b.float()
    return a.shape == b.shape and torch.allclose(a, b, atol=rtol, rtol=rtol, equal_nan=True)


def _perm(n: int, device, seed: int = 17) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randperm(n, generator=g).to(device)


def _same_shape(xs) -> List[int]:
    return [i for i, x in enumerate(xs) if torch.is_tensor(x) and x.shape == xs[0].shape]


def elementwise_permutation(fn: Callable, *xs: torch.Tensor, rtol: float = 1e-2) -> Tuple[bool, str]:
    n = xs[0].numel()
    p = _perm(n, xs[0].device)
    idx = _same_shape(xs)
    y = fn(*xs).reshape(-1)
    xp = [x.reshape(-1)[p].reshape(x.shape) if i in idx else x for i, x in enumerate(xs)]
    return _close(y[p], fn(*xp).reshape(-1), rtol), "elementwise permutation equivariance"


def elementwise_locality(fn: Callable, *xs: torch.Tensor, rtol: float = 1e-2) -> Tuple[bool, str]:
    y = fn(*xs).reshape(-1)
    xs2 = [x.clone() for x in xs]
    i = xs[0].numel() // 2
    xs2[0].view(-1)[i] += 1.0
    y2 = fn(*xs2).reshape(-1)
    mask = torch.ones_like(y, dtype=torch.bool)
    mask[i] = False
    return _close(y[mask], y2[mask], rtol), "only the perturbed element may change"


def elementwise_reshape(fn: Callable, *xs: torch.Tensor, rtol: float = 1e-2) -> Tuple[bool, str]:
    x0 = xs[0]
    if x0.dim() < 2 or x0.shape[-1] % 2:
        return True, "reshape invariance (not applicable)"
    idx = _same_shape(xs)
    shp = (*x0.shape[:-1], 2, x0.shape[-1] // 2)
    try:
        y2 = fn(*[x.reshape(shp) if i in idx else x for i, x in enumerate(xs)]).reshape(x0.shape)
    except Exception:  # noqa: BLE001 - an entry point tied to 2-D inputs: not applicable
        return True, "reshape invariance (not applicable)"
    return _close(fn(*xs), y2, rtol), "reshape invariance"


def reduction_row_permutation(fn: Callable, x: torch.Tensor, *rest, rtol: float = 1e-2) -> Tuple[bool, str]:
    p = _perm(x.shape[0], x.device)
    return _close(fn(x, *rest)[p], fn(x[p], *rest), rtol), "row permutation equivariance"


def reduction_row_locality(fn: Callable, x: torch.Tensor, *rest, rtol: float = 1e-2) -> Tuple[bool, str]:
    y = fn(x, *rest)
    x2 = x.clone()
    r = x.shape[0] // 2
    x2[r] = x2[r] * 0.5 + 0.25
    y2 = fn(x2, *rest)
    keep = torch.ones(x.shape[0], dtype=torch.bool, device=x.device)
    keep[r] = False
    return _close(y[keep], y2[keep], rtol), "only the perturbed row may change"


def reduction_inrow_permutation(fn: Callable, x: torch.Tensor, *rest, rtol: float = 1e-2) -> Tuple[bool, str]:
    p = _perm(x.shape[-1], x.device, seed=29)
    rest_p = [t[..., p] if torch.is_tensor(t) and t.dim() >= 1 and t.shape[-1] == x.shape[-1] else t for t in rest]
    y, yp = fn(x, *rest), fn(x[..., p], *rest_p)
    if y.shape == x.shape:
        return _close(y[..., p], yp, rtol), "in-row permutation equivariance"
    return _close(y, yp, rtol), "in-row permutation invariance"


def relations_for(op_class: str) -> List[Callable]:
    c = (op_class or "").lower()
    if any(k in c for k in ELEMENTWISE):
        return [elementwise_permutation, elementwise_locality, elementwise_reshape]
    if any(k in c for k in REDUCTION):
        return [reduction_row_permutation, reduction_row_locality, reduction_inrow_permutation]
    return []
