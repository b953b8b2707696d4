"""Free Viewpoint Matching (FVM), Eq. (13) of the JEANIE paper, on B200 kernels.

Semantics of hibana2077/torchwarp src/torchwarp/jeanie/fvm.py:15-67: a
viewpoint soft-min at every temporal pair (native kernel), then soft-DTW on
the result (native DP).
"""

import torch

from .. import sdtw
from ..udtw.functional import _BACKENDS, _check_backend
from .. import _transforms
from . import _ops
from .distances import euclidean_cost, rbf_cost, squared_euclidean_cost

_METRICS = {"euclidean": euclidean_cost, "sqeuclidean": squared_euclidean_cost,
            "rbf": rbf_cost}


def _check_backend_name(backend):
    """The backend check of soft_dtw_from_cost (sdtw.py), for the fused path
    that does not go through it."""
    if backend not in _BACKENDS:
        raise ValueError("backend must be one of {}".format(_BACKENDS))
    _check_backend(backend)


def fvm_from_cost(cost, *, gamma=0.1, backend="auto"):
    """FVM on a precomputed cost [B, K..., T, U] (every dim between B and
    [T, U] is a viewpoint index reduced by the soft-min); returns [B]."""
    if not cost.is_floating_point():
        raise TypeError("cost must be a floating-point tensor")
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if cost.ndim < 4:
        raise ValueError("cost must be [B, K..., T, U] with at least one viewpoint dim")
    B, T, U = cost.shape[0], cost.shape[-2], cost.shape[-1]
    K = 1
    for k in cost.shape[1:-2]:
        K *= k
    flat = cost.reshape(B, K, T, U)
    if flat.dtype not in (torch.float32, torch.float64):
        flat = flat.float()
    _check_backend_name(backend)
    if flat.dtype == torch.float32 and min(K, T, U) > 0 and \
            _ops.fused_supported(K, T, U, 0, True, False):
        # viewpoint soft-min and soft-DTW in one native call per direction
        return _ops.fused_apply(None, None, flat, K, 1, T, U, 0, 0, gamma, 0, True, False)[0]
    temporal = _transforms.pick(_ops.FvmSoftmin, _ops.FvmSoftminTraced).apply(flat, float(gamma))
    return sdtw.soft_dtw_from_cost(temporal, gamma=gamma, backend=backend)


def fvm(query, support, *, gamma=0.1, metric="euclidean", backend="auto"):
    """FVM between query [B, K..., T, D] and support [B, U, D] or [B, K'..., U, D]."""
    if metric not in _METRICS:
        raise ValueError("metric must be one of {}".format(tuple(_METRICS)))
    if query.ndim < 4 or support.ndim < 3:
        raise ValueError("query must be [B, K..., T, D] and support [B, U, D] or "
                         "[B, K'..., U, D]")
    B, T, D = query.shape[0], query.shape[-2], query.shape[-1]
    U = support.shape[-2]
    K = 1
    for k in query.shape[1:-2]:
        K *= k
    q = query.reshape(B, K, T, D)
    if support.ndim == 3:
        K = q.shape[1]
        dtype = torch.promote_types(query.dtype, support.dtype)
        dtype = dtype if dtype in (torch.float32, torch.float64) else torch.float32
        if metric != "rbf" and dtype == torch.float32 and gamma > 0 and \
                support.shape[0] == B and support.shape[-1] == D and min(K, T, U) > 0 and \
                _ops.fused_supported(K, T, U, D, True, True):
            _check_backend_name(backend)
            # cost, viewpoint soft-min, soft-DTW and their backward on chip:
            # the [B, K, T, U] cost never reaches HBM as a separate tensor
            return _ops.fused_apply(q.to(torch.float32).reshape(B, K * T, D),
                                    support.to(torch.float32), None, K, 1, T, U, 0, 0, gamma,
                                    1 if metric == "euclidean" else 0, True, False)[0]
        cost = _METRICS[metric](q, support)                      # [B, K, T, U]
    else:
        # Every (query viewpoint, support viewpoint) pair: all K' U support
        # frames of a pair form one support set of the query/support kernel,
        # [B, K T, K' U], instead of expanding the query K' times and the
        # support K times; one permute of the (small) cost gives the
        # reference's [B, K, K', T, U] (jeanie/fvm.py:62-66).
        K = q.shape[1]
        Kp = 1
        for k in support.shape[1:-2]:
            Kp *= k
        s = support.reshape(B, Kp, U, D)
        Kp = s.shape[1]
        full = _METRICS[metric](q.reshape(B, K * T, D), s.reshape(B, Kp * U, D))
        cost = full.reshape(B, K, T, Kp, U).permute(0, 1, 3, 2, 4)
    return fvm_from_cost(cost, gamma=gamma, backend=backend)
