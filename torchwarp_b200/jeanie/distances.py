"""Batched base distances (cost tensors) for uDTW, JEANIE, FVM and soft-DTW.

Semantics of hibana2077/torchwarp src/torchwarp/jeanie/distances.py:1-51.
Two layouts:
  JEANIE / FVM:  query [..., K, T, D], support [..., U, D] -> [..., K, T, U]
                 (support has the same leading batch dims as query, or none)
  two sequences: x [..., N, D], y [..., M, D] (same rank) -> [..., N, M]
The (squared) Euclidean distances run in the native query/support cost kernel
(GEMM form |q|^2 + |s|^2 - 2 q.s, clamped at 0; the Euclidean root has zero
gradient at 0).  ``rbf_cost`` has no GEMM form; it runs in its own native
kernel, which sums over the features per (frame, frame) pair instead of
materialising the [..., T, U, D] difference tensor of the reference's
PyTorch expression.
"""

import torch

from .. import _transforms
from . import _ops


def _check(query, support):
    if support.ndim < 2 or query.ndim < support.ndim:
        raise ValueError("query must be [..., K, T, D] or [..., N, D] and support "
                         "[..., U, D] or [..., M, D]")
    if query.shape[-1] != support.shape[-1]:
        raise ValueError("query/support feature dimensions do not match")
    return support.unsqueeze(-3) if query.ndim > support.ndim else support


def _native_cost(query, support, metric, sigma=None):
    """Flatten to query rows [L, R, D] against supports [L, U, D], run the kernel
    (the rbf kernel when sigma is given)."""
    dtype = torch.promote_types(query.dtype, support.dtype)
    if dtype not in (torch.float32, torch.float64):
        dtype = torch.float32
    bcast = query.ndim > support.ndim
    s = support.unsqueeze(-3) if bcast else support
    lead = torch.broadcast_shapes(query.shape[:-3 if bcast else -2], s.shape[:-3 if bcast else -2])
    D = query.shape[-1]
    if bcast:
        K, T = query.shape[-3], query.shape[-2]
        U = support.shape[-2]
        q = query.to(dtype).expand(*lead, K, T, D).reshape(-1, K * T, D)
        sp = support.to(dtype).expand(*lead, U, D).reshape(-1, U, D)
        out = _apply(q, sp, metric, sigma)
        return out.reshape(*lead, K, T, U)
    N, M = query.shape[-2], support.shape[-2]
    q = query.to(dtype).expand(*lead, N, D).reshape(-1, N, D)
    sp = support.to(dtype).expand(*lead, M, D).reshape(-1, M, D)
    return _apply(q, sp, metric, sigma).reshape(*lead, N, M)


def _apply(q, sp, metric, sigma):
    if sigma is not None:
        return _ops.QSRbfCost.apply(q, sp, float(sigma))
    return _transforms.pick(_ops.QSCost, _ops.QSCostTraced).apply(q, sp, metric)


def squared_euclidean_cost(query: torch.Tensor, support: torch.Tensor) -> torch.Tensor:
    """Squared-Euclidean base distance."""
    _check(query, support)
    return _native_cost(query, support, 0)


def euclidean_cost(query: torch.Tensor, support: torch.Tensor) -> torch.Tensor:
    """Euclidean base distance; the gradient at zero distance is 0."""
    _check(query, support)
    return _native_cost(query, support, 1)


def rbf_cost(query: torch.Tensor, support: torch.Tensor, sigma: float = 0.5) -> torch.Tensor:
    """RBF-style base cost d(x,y) = sum_d [2 - 2 exp(-sigma (x_d - y_d)^2)].

    The per-dimension form has no matmul; the native kernel sums it per
    (frame, frame) pair without the [..., K, T, U, D] difference tensor.
    """
    if sigma <= 0:
        raise ValueError("sigma must be > 0")
    _check(query, support)
    return _native_cost(query, support, None, sigma)
