"""Metamorphic relations: properties an implementation must satisfy without
an oracle (reference parity: kore/verify/metamorphic.py:183-205).

* elementwise ops commute with permutations of the flattened input and
  compute each element from its own position only (locality);
* row reductions are invariant to permutations inside a row and
  equivariant to row permutations;
* reshape invariance for elementwise ops.
Each check returns (ok, detail)."""
from __future__ import annotations

from typing import Callable, Tuple

import torch


def _close(a, b, tol=1e-2) -> bool:
    return torch.allclose(a.float(), b.float(), atol=tol, rtol=tol)


def elementwise_permutation(fn: Callable, *xs: torch.Tensor) -> Tuple[bool, str]:
    n = xs[0].numel()
    perm = torch.randperm(n, device=xs[0].device)
    y = fn(*xs).reshape(-1)
    yp = fn(*[x.reshape(-1)[perm].reshape(x.shape) for x in xs]).reshape(-1)
    return _close(y[perm], yp), "elementwise permutation equivariance"


def elementwise_locality(fn: Callable, *xs: torch.Tensor) -> Tuple[bool, str]:
    y = fn(*xs).reshape(-1)
    xs2 = [x.clone() for x in xs]
    i = xs[0].numel() // 2
    xs2[0].view(-1)[i] += 1.0
    y2 = fn(*xs2).reshape(-1)
    mask = torch.ones_like(y, dtype=torch.bool)
    mask[i] = False
    return _close(y[mask], y2[mask]), "only the perturbed element may change"


def reduction_row_permutation(fn: Callable, x: torch.Tensor, *rest) -> Tuple[bool, str]:
    perm = torch.randperm(x.shape[0], device=x.device)
    return _close(fn(x, *rest)[perm], fn(x[perm], *rest)), "row permutation equivariance"


def reduction_inrow_permutation(fn: Callable, x: torch.Tensor, *rest) -> Tuple[bool, str]:
    """For reductions whose output is a per-row scalar or is permuted with the row."""
    perm = torch.randperm(x.shape[-1], device=x.device)
    y, yp = fn(x, *rest), fn(x[..., perm], *rest)
    if y.shape == x.shape:
        return _close(y[..., perm], yp), "in-row permutation equivariance"
    return _close(y, yp), "in-row permutation invariance"
