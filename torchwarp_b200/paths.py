"""Alignment paths, in the notation of the uDTW and JEANIE papers.

Semantics of hibana2077/torchwarp src/torchwarp/paths.py:1-201:
* ``path_matrix``: the soft-min-weighted path matrices (uDTW Eq. 3), equal to
  the gradient of the distance with respect to the cost; computed here by the
  native backward kernels.
* ``optimal_path``: the path with the smallest cost (gamma -> 0), from the
  native float64 kernel with the reference's tie-break order, so the cells
  are identical to the reference's.
Plotting (``torchwarp.plot`` in the reference) is not part of this package.
"""

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch

from . import _native as nat
from .jeanie import euclidean_cost, fvm_from_cost, jeanie_from_cost, squared_euclidean_cost
from .sdtw import soft_dtw_from_cost
from .udtw import pairwise_matrices, udtw_from_cost

__all__ = ["Alignment", "soft_dtw", "soft_dtw_per_view", "udtw", "fvm", "jeanie", "optimal_path"]


@dataclass
class Alignment:
    """Result of a path computation (batched over the first dimension).

    Attributes:
        distance: [B] distance d.
        path_matrix: [B, T, U] (or [B, K, T, U]) soft-min-selected path matrices.
        optimal_path: per batch item, the cells (t, u) (or (t, u, k)) of the
            path with the smallest distance, from (0, 0) to (T-1, U-1).
        cost: the cost tensor the paths are evaluated on (uDTW: D / Sigma).
        Sigma: [B, T, U] pair-wise variances (uDTW only).
        Omega: [B] penalty times beta (uDTW only).
        angles: viewpoint labels for the K axis, if given.
    """

    distance: torch.Tensor
    path_matrix: torch.Tensor
    optimal_path: List[List[Tuple[int, ...]]]
    cost: torch.Tensor
    Sigma: Optional[torch.Tensor] = None
    Omega: Optional[torch.Tensor] = None
    angles: Optional[list] = field(default=None)

    def plot(self, type="alignment", **kwargs):
        raise NotImplementedError("plotting is not part of torchwarp_b200")


def _value_and_grad(fn, D):
    with torch.enable_grad():
        c = D.detach().clone().requires_grad_(True)
        d = fn(c)
        (g,) = torch.autograd.grad(d.sum(), c)
    return d.detach(), g.detach()


def _optimal(cost, max_shift, start_view):
    """cost [B, K, T, U] -> list of (t, u, k) paths (native float64 kernel)."""
    nat.require_cuda(cost)
    B, K, T, U = cost.shape
    D = cost.detach().to(torch.float64).contiguous()
    r = torch.empty_like(D)
    back = torch.empty(D.shape, dtype=torch.int32, device=D.device)
    path = torch.empty(B, T + U - 1, 3, dtype=torch.int32, device=D.device)
    length = torch.empty(B, dtype=torch.int32, device=D.device)
    if B:
        with torch.cuda.device(D.device):
            nat.check(nat.call("optimal_path", nat.lib().tw_optimal_path_f64, nat.ptr(D), B, K, T,
                               U, int(max_shift), -1 if start_view is None else int(start_view),
                               nat.ptr(r), nat.ptr(back), nat.ptr(path), nat.ptr(length),
                               nat.stream_of(D)), "tw_optimal_path")
    p, n = path.cpu().tolist(), length.cpu().tolist()
    return [[tuple(c) for c in p[b][:n[b]]] for b in range(B)]


def optimal_path(cost, *, max_shift=0, start_view=None):
    """Paths with the smallest distance for a batch of cost matrices.

    cost: [B, T, U] (cells (t, u)) or [B, K, T, U] (cells (t, u, k)).
    """
    if cost.ndim == 3:
        return [[(t, u) for t, u, _ in p] for p in _optimal(cost.unsqueeze(1), 0, None)]
    return _optimal(cost, max_shift, start_view)


def _base_distance(query, support, metric):
    if metric == "euclidean":
        return euclidean_cost(query, support)
    if metric == "sqeuclidean":
        return squared_euclidean_cost(query, support)
    raise ValueError("metric must be 'euclidean' or 'sqeuclidean'")


def soft_dtw(cost, *, gamma=0.1):
    """soft-DTW paths for a cost matrix [B, T, U]."""
    d, pm = _value_and_grad(lambda x: soft_dtw_from_cost(x, gamma=gamma), cost)
    return Alignment(d, pm, optimal_path(cost), cost)


def soft_dtw_per_view(query, support, *, gamma=0.1, metric="euclidean", angles=None):
    """soft-DTW with each viewpoint of the query aligned separately; query
    [B, K, T, d], support [B, U, d]; returns K Alignments with cells (t, u, k)."""
    D = _base_distance(query, support, metric)
    out = []
    for k in range(D.shape[1]):
        a = soft_dtw(D[:, k], gamma=gamma)
        a.optimal_path = [[(t, u, k) for t, u in p] for p in a.optimal_path]
        a.angles = angles
        out.append(a)
    return out


def udtw(X, Y, sigma_x, sigma_y, *, gamma=1.0, beta=1.0):
    """uDTW paths (evaluated on D * Sigma^dagger, uDTW Eq. 2)."""
    with torch.no_grad():
        DS, pen, Sigma = pairwise_matrices(X, Y, sigma_x, sigma_y, beta)
    d, pm = _value_and_grad(lambda x: udtw_from_cost(x, pen, gamma=gamma).distance, DS)
    with torch.no_grad():
        Omega = udtw_from_cost(DS, pen, gamma=gamma).penalty
    return Alignment(d, pm, optimal_path(DS), DS, Sigma=Sigma, Omega=Omega)


def fvm(query, support, *, gamma=0.1, metric="euclidean", angles=None):
    """FVM paths (query viewpoints only); the viewpoint is free at each step."""
    D = _base_distance(query, support, metric)
    d, pm = _value_and_grad(lambda x: fvm_from_cost(x, gamma=gamma), D)
    return Alignment(d, pm, optimal_path(D, max_shift=D.shape[1]), D, angles=angles)


def jeanie(query, support, *, gamma=0.1, max_shift=1, metric="euclidean", angles=None,
           start_view=None):
    """JEANIE paths (one viewpoint axis); ``start_view`` restricts the paths to
    start at that viewpoint (JEANIE Fig. 7)."""
    D = _base_distance(query, support, metric)
    Ds = D
    if start_view is not None:
        block = torch.zeros_like(D)
        block[:, :, 0, 0] = 1e4
        block[:, start_view, 0, 0] = 0
        Ds = D + block
    d, pm = _value_and_grad(lambda x: jeanie_from_cost(x, gamma=gamma, max_shift=max_shift), Ds)
    return Alignment(d, pm, optimal_path(D, max_shift=max_shift, start_view=start_view), D,
                     angles=angles)
