"""Batched base distances (cost tensors) for uDTW, JEANIE, FVM and soft-DTW.

Semantics of hibana2077/torchwarp src/torchwarp/jeanie/distances.py:1-51.
Two layouts:
  JEANIE / FVM:  query [..., K, T, D], support [..., U, D] -> [..., K, T, U]
                 (support has the same leading batch dims as query, or none)
  two sequences: x [..., N, D], y [..., M, D] (same rank) -> [..., N, M]
The (squared) Euclidean distances run in the native query/support cost kernel
(GEMM form |q|^2 + |s|^2 - 2 q.s, clamped at 0; the Euclidean root has zero
gradient at 0).  ``rbf_cost`` has no GEMM form and stays a PyTorch
expression, as in the reference.
"""

import torch

from . import _ops


def _check(query, support):
    if support.ndim < 2 or query.ndim < support.ndim:
        raise ValueError("query must be [..., K, T, D] or [..., N, D] and support "
                         "[..., U, D] or [..., M, D]")
    if query.shape[-1] != support.shape[-1]:
        raise ValueError("query/support feature dimensions do not match")
    return support.unsqueeze(-3) if query.ndim > support.ndim else support


def _native_cost(query, support, metric):
    """Flatten to query rows [L, R, D] against supports [L, U, D], run the kernel."""
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
        out = _ops.QSCost.apply(q, sp, metric)
        return out.reshape(*lead, K, T, U)
    N, M = query.shape[-2], support.shape[-2]
    q = query.to(dtype).expand(*lead, N, D).reshape(-1, N, D)
    sp = support.to(dtype).expand(*lead, M, D).reshape(-1, M, D)
    return _ops.QSCost.apply(q, sp, metric).reshape(*lead, N, M)


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

    This per-dimension form cannot be written as a matmul, so it
    materialises the [..., K, T, U, D] difference tensor.
    """
    if sigma <= 0:
        raise ValueError("sigma must be > 0")
    s = _check(query, support)
    diff = query.unsqueeze(-2) - s.unsqueeze(-3)
    return (2.0 - 2.0 * torch.exp(-sigma * diff.pow(2))).sum(dim=-1)
