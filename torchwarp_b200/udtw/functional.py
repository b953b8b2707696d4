"""Uncertainty-DTW (uDTW, Wang & Koniusz, ECCV 2022) on B200 kernels.

Same public semantics as hibana2077/torchwarp src/torchwarp/udtw/functional.py
(validation :34-101, ``udtw_from_cost`` :104-144, ``udtw`` :166-209):
  Sigma_ij = max(0.5 (sigma_i^2 + sigma'_j^2), eps)      (Eq. 8)
  cost_ij  = |x_i - y_j|^2 / Sigma_ij, penalty_ij = beta log Sigma_ij (Eq. 16)
  distance = soft-min path cost, penalty = soft-min-weighted penalty (Eq. 3).
The DP and the cost construction run in the native sm_100a library; CPU
tensors are rejected.  ``backend`` accepts "auto" and "cuda" (both native);
"torch" is not available in this build.
"""

from typing import NamedTuple

import torch

from . import _ops

_BACKENDS = ("auto", "cuda", "torch")


class UDTWOutput(NamedTuple):
    """Result of uDTW: ``distance`` [B] and the beta-weighted ``penalty`` [B].

    A tuple, so ``d, omega = ...`` also works.
    """

    distance: torch.Tensor
    penalty: torch.Tensor


def _check_backend(backend):
    if backend not in _BACKENDS:
        raise ValueError("backend must be one of {}".format(_BACKENDS))
    if backend == "torch":
        raise RuntimeError("torchwarp_b200 has no PyTorch (CPU) backend; use backend='auto' or "
                           "'cuda' with CUDA tensors")


def _check_sequence_inputs(X, Y, sigma_x, sigma_y):
    if X.ndim != 3 or Y.ndim != 3:
        raise ValueError("X and Y must have shape [batch, time, feature]")
    if sigma_x.ndim != 3 or sigma_y.ndim != 3:
        raise ValueError("the uncertainties sigma must have shape [batch, time, 1]")
    if X.shape[0] != Y.shape[0]:
        raise ValueError("X and Y must have the same batch size")
    if X.shape[2] != Y.shape[2]:
        raise ValueError("X and Y must have the same feature dimension")
    if sigma_x.shape[:2] != X.shape[:2] or sigma_y.shape[:2] != Y.shape[:2]:
        raise ValueError("uncertainty tensors must match batch/time dimensions")
    if sigma_x.shape[2] != 1 or sigma_y.shape[2] != 1:
        raise ValueError("the uncertainties sigma must have shape [batch, time, 1]")
    if not X.is_floating_point() or not Y.is_floating_point():
        raise TypeError("X and Y must be floating-point tensors")
    if not sigma_x.is_floating_point() or not sigma_y.is_floating_point():
        raise TypeError("the uncertainties sigma must be floating-point tensors")


def _check_hyperparameters(gamma, beta, bandwidth):
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if beta < 0:
        raise ValueError("beta must be >= 0")
    if bandwidth is not None and bandwidth < 0:
        raise ValueError("bandwidth must be None or >= 0")


def _squared_euclidean(X, Y, method="gemm"):
    """Pairwise squared distances [B,N,M] (GEMM form, or materialised difference)."""
    if method == "diff":
        return (X.unsqueeze(2) - Y.unsqueeze(1)).pow(2).sum(dim=3)
    if method != "gemm":
        raise ValueError("method must be 'gemm' or 'diff'")
    x2 = X.pow(2).sum(-1, keepdim=True)
    y2 = Y.pow(2).sum(-1).unsqueeze(1)
    return torch.baddbmm(x2 + y2, X, Y.transpose(1, 2), alpha=-2.0).clamp_min(0)


def pairwise_matrices(X, Y, sigma_x, sigma_y, beta=1.0, eps=1e-8, *, method="gemm"):
    """Uncertainty-weighted cost, beta-weighted log-variance penalty, variance.

    Eq. (8):  Sigma_ij = 0.5 * (sigma_i^2 + sigma'_j^2)
    Eq. (16): cost_ij = ||x_i - y_j||^2 / Sigma_ij, penalty_ij = beta * log Sigma_ij
    """
    _check_sequence_inputs(X, Y, sigma_x, sigma_y)
    if eps <= 0:
        raise ValueError("eps must be > 0")
    if beta < 0:
        raise ValueError("beta must be >= 0")
    variance = (0.5 * (sigma_x.pow(2) + sigma_y.pow(2).transpose(1, 2))).clamp_min(eps)
    weighted_cost = _squared_euclidean(X, Y, method) / variance
    weighted_penalty = beta * torch.log(variance)
    return weighted_cost, weighted_penalty, variance


def _check_band_reached(distance, band):
    # A data-dependent check (one host sync); skipped while torch.compile traces.
    if band > 0 and not torch.compiler.is_compiling():
        if not bool(torch.isfinite(distance).all()):
            raise ValueError("No valid DTW path reaches the final cell under the given bandwidth")


def _float(t):
    return t if t.dtype in (torch.float32, torch.float64) else t.float()


def udtw_from_cost(cost, penalty, *, gamma=1.0, bandwidth=None, backend="auto"):
    """Run the uDTW dynamic program on precomputed matrices.

    Args:
        cost: [B,N,M] uncertainty-weighted cost, e.g. D / Sigma.
        penalty: [B,N,M] per-cell penalty, e.g. beta * log Sigma.
        gamma: SoftMin temperature (> 0).
        bandwidth: Sakoe-Chiba band; None or 0 disables pruning.
        backend: "auto" or "cuda" (native kernels).

    Returns:
        UDTWOutput(distance [B], penalty [B]).
    """
    if cost.ndim != 3 or penalty.ndim != 3:
        raise ValueError("cost and penalty must have shape [B,N,M]")
    if cost.shape != penalty.shape:
        raise ValueError("cost and penalty must have identical shapes")
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if bandwidth is not None and bandwidth < 0:
        raise ValueError("bandwidth must be None or >= 0")
    _check_backend(backend)
    if cost.shape[1] == 0 or cost.shape[2] == 0:
        raise ValueError("sequence lengths must be non-zero")
    cost, penalty = _float(cost), _float(penalty)
    if penalty.dtype != cost.dtype:
        penalty = penalty.to(cost.dtype)
    # The recurrence and the band are symmetric in (i, j); the kernels stream
    # the longer sequence, so keep N <= M.
    if cost.shape[1] > cost.shape[2]:
        cost, penalty = cost.transpose(1, 2), penalty.transpose(1, 2)
    band = 0.0 if bandwidth is None else float(bandwidth)
    distance, pen, _ = _ops.dp_apply(cost, penalty, float(gamma), band)
    _check_band_reached(distance, band)
    return UDTWOutput(distance, pen)


def _udtw_fused(X, Y, sigma_x, sigma_y, beta, gamma, bandwidth, eps):
    """uDTW with the cost and penalty built by the native cost kernel."""
    if X.shape[1] > Y.shape[1]:
        X, Y, sigma_x, sigma_y = Y, X, sigma_y, sigma_x
    dtype = X.dtype if X.dtype in (torch.float32, torch.float64) else torch.float32
    X, Y = X.to(dtype), Y.to(dtype)
    vx = None if sigma_x is None else sigma_x.squeeze(-1).to(dtype).pow(2)
    vy = None if sigma_y is None else sigma_y.squeeze(-1).to(dtype).pow(2)
    band = 0.0 if bandwidth is None else float(bandwidth)
    distance, pen, _, _ = _ops.fused_apply(X, Y, vx, vy, float(gamma), float(beta), float(eps),
                                          band)
    _check_band_reached(distance, band)
    return UDTWOutput(distance, pen)


def _sdtw_fused(X, Y, gamma, bandwidth):
    """soft-DTW distance with the squared-Euclidean cost built natively (uDTW
    with unit variance and no penalty, sdtw.py:78-84); the backward keeps the
    cost's positivity mask instead of the cost."""
    if X.shape[1] > Y.shape[1]:
        X, Y = Y, X
    dtype = X.dtype if X.dtype in (torch.float32, torch.float64) else torch.float32
    X, Y = X.to(dtype), Y.to(dtype)
    band = 0.0 if bandwidth is None else float(bandwidth)
    distance, _, _ = _ops.sdtw_fused_apply(X, Y, float(gamma), band)
    _check_band_reached(distance, band)
    return distance


def udtw(X, Y, sigma_x, sigma_y, *, beta=1.0, gamma=1.0, normalize=False, bandwidth=None,
         method="gemm", eps=1e-8, backend="auto"):
    """Uncertainty-DTW between two batches of sequences.

    Args:
        X, Y: [B,N,D], [B,M,D] sequences.
        sigma_x, sigma_y: [B,N,1], [B,M,1] positive standard deviations.
        beta: Penalty weight (>= 0).
        gamma: SoftMin temperature (> 0).
        normalize: If True, return d(X,Y) - 0.5 [d(X,X) + d(Y,Y)] for both
            the distance and the penalty.
        bandwidth: Sakoe-Chiba band; None or 0 disables pruning.
        method: "gemm" (cost built by the native kernel from the features) or
            "diff" (materialised matrices, see ``pairwise_matrices``).
        eps: Lower bound applied to the variance.
        backend: "auto" or "cuda" (native kernels).

    Returns:
        UDTWOutput(distance [B], penalty [B]); the penalty is beta-weighted.
    """
    _check_sequence_inputs(X, Y, sigma_x, sigma_y)
    _check_hyperparameters(gamma, beta, bandwidth)
    if eps <= 0:
        raise ValueError("eps must be > 0")
    if method not in ("gemm", "diff"):
        raise ValueError("method must be 'gemm' or 'diff'")
    _check_backend(backend)
    if X.shape[1] == 0 or Y.shape[1] == 0:
        raise ValueError("sequence lengths must be non-zero")

    def run(A, Bq, sa, sb):
        if method == "gemm":
            return _udtw_fused(A, Bq, sa, sb, beta, gamma, bandwidth, eps)
        cost, pen, _ = pairwise_matrices(A, Bq, sa, sb, beta, eps, method=method)
        return udtw_from_cost(cost, pen, gamma=gamma, bandwidth=bandwidth, backend=backend)

    d_xy, p_xy = run(X, Y, sigma_x, sigma_y)
    if not normalize:
        return UDTWOutput(d_xy, p_xy)
    d_xx, p_xx = run(X, X, sigma_x, sigma_x)
    d_yy, p_yy = run(Y, Y, sigma_y, sigma_y)
    return UDTWOutput(d_xy - 0.5 * (d_xx + d_yy), p_xy - 0.5 * (p_xx + p_yy))
