"""soft-DTW (Cuturi & Blondel, ICML 2017) on B200 kernels.

Semantics of hibana2077/torchwarp src/torchwarp/sdtw.py:12-136.  soft-DTW is
uDTW with unit variance and no penalty: ``soft_dtw`` builds the squared
Euclidean cost with the native cost kernel and runs the native DP;
``soft_dtw_from_cost`` runs the same DP on a given cost (the reference
routes it through its JEANIE kernel with one viewpoint, or through its uDTW
kernel when a band is set; the recurrence is the same).
"""

from typing import Optional

import torch
import torch.nn as nn

from .udtw import _ops as _udtw_ops
from .udtw.functional import (_BACKENDS, _check_backend, _check_band_reached, _float,
                              _sdtw_fused, udtw_from_cost)


def softmin(x: torch.Tensor, gamma: float, dim: Optional[int] = None) -> torch.Tensor:
    """Differentiable soft minimum -gamma * logsumexp(-x / gamma)."""
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if dim is None:
        x = x.reshape(-1)
        dim = 0
    return -gamma * torch.logsumexp(-x / gamma, dim=dim)


def softmin_weights(values: torch.Tensor, gamma: float, dim: int = 0) -> torch.Tensor:
    """Weights of the soft minimum, softmax(-values / gamma) over ``dim``."""
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    return torch.softmax(-values / gamma, dim=dim)


def soft_dtw_from_cost(cost: torch.Tensor, *, gamma: float = 1.0,
                       bandwidth: Optional[float] = None, backend: str = "auto") -> torch.Tensor:
    """soft-DTW on a precomputed cost [B, T, U]; returns [B].

    Args:
        cost: [B, T, U] cost matrices.
        gamma: SoftMin temperature (> 0).
        bandwidth: Sakoe-Chiba band; None or 0 disables pruning.
        backend: "auto" or "cuda" (native kernels).
    """
    if not cost.is_floating_point():
        raise TypeError("cost must be a floating-point tensor")
    if cost.ndim != 3:
        raise ValueError("cost must have shape [B, T, U]")
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if bandwidth is not None and bandwidth < 0:
        raise ValueError("bandwidth must be None or >= 0")
    _check_backend(backend)
    if min(cost.shape[1], cost.shape[2]) == 0:
        raise ValueError("cost dimensions must be non-empty")
    cost = _float(cost)
    if cost.shape[1] > cost.shape[2]:
        cost = cost.transpose(1, 2)
    band = 0.0 if not bandwidth else float(bandwidth)
    distance, _, _ = _udtw_ops.dp_apply(cost, None, float(gamma), band)
    _check_band_reached(distance, band)
    return distance


def soft_dtw(X: torch.Tensor, Y: torch.Tensor, *, gamma: float = 1.0, normalize: bool = False,
             bandwidth: Optional[float] = None, dist_func=None,
             backend: str = "auto") -> torch.Tensor:
    """soft-DTW between two batches of sequences.

    Args:
        X, Y: [B,N,D], [B,M,D] sequences.
        gamma: SoftMin temperature (> 0).
        normalize: If True, return the soft-DTW divergence
            d(X,Y) - 0.5 [d(X,X) + d(Y,Y)].
        bandwidth: Sakoe-Chiba band; None or 0 disables pruning.
        dist_func: Optional function (X, Y) -> cost [B,N,M].  Default: squared
            Euclidean distance, built by the native cost kernel.
        backend: "auto" or "cuda" (native kernels).

    Returns:
        distance [B]
    """
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if bandwidth is not None and bandwidth < 0:
        raise ValueError("bandwidth must be None or >= 0")
    if backend not in _BACKENDS:
        raise ValueError("backend must be one of {}".format(_BACKENDS))
    if X.ndim != 3 or Y.ndim != 3:
        raise ValueError("X and Y must have shape [batch, time, feature]")
    _check_backend(backend)

    def run(A, Bq):
        if dist_func is None:
            if A.shape[0] != Bq.shape[0] or A.shape[2] != Bq.shape[2]:
                raise ValueError("X and Y must have the same batch size and feature dimension")
            if not A.is_floating_point() or not Bq.is_floating_point():
                raise TypeError("X and Y must be floating-point tensors")
            if A.shape[1] == 0 or Bq.shape[1] == 0:
                raise ValueError("sequence lengths must be non-zero")
            # unit variance, no penalty: cost = max(|x|^2 + |y|^2 - 2 x.y, 0)
            return _sdtw_fused(A, Bq, gamma, bandwidth)
        cost = dist_func(A, Bq)
        return udtw_from_cost(cost, torch.zeros_like(cost), gamma=gamma, bandwidth=bandwidth,
                              backend=backend).distance

    d = run(X, Y)
    if not normalize:
        return d
    return d - 0.5 * (run(X, X) + run(Y, Y))


class SoftDTW(nn.Module):
    """soft-DTW module; see ``torchwarp_b200.functional.soft_dtw``.

    Args:
        gamma: SoftMin temperature (> 0).
        normalize: If True, return the soft-DTW divergence
            d(X,Y) - 0.5 [d(X,X) + d(Y,Y)].
        bandwidth: Sakoe-Chiba band; None or 0 disables pruning.
        dist_func: Optional function (X, Y) -> cost [B,N,M].
        backend: "auto" or "cuda".

    Forward:
        X, Y: [B,N,D], [B,M,D]

    Returns:
        distance [B]
    """

    def __init__(self, gamma=1.0, normalize=False, bandwidth=None, dist_func=None, *,
                 backend="auto"):
        super().__init__()
        if gamma <= 0:
            raise ValueError("gamma must be > 0")
        if bandwidth is not None and bandwidth < 0:
            raise ValueError("bandwidth must be None or >= 0")
        if backend not in _BACKENDS:
            raise ValueError("backend must be one of {}".format(_BACKENDS))
        self.gamma = float(gamma)
        self.normalize = bool(normalize)
        self.bandwidth = None if bandwidth is None else float(bandwidth)
        self.dist_func = dist_func
        self.backend = backend

    def forward(self, X, Y):
        return soft_dtw(X, Y, gamma=self.gamma, normalize=self.normalize,
                        bandwidth=self.bandwidth, dist_func=self.dist_func, backend=self.backend)

    def extra_repr(self):
        return "gamma={}, normalize={}, bandwidth={}, backend={!r}".format(
            self.gamma, self.normalize, self.bandwidth, self.backend)
