"""JEANIE temporal-viewpoint alignment on B200 kernels.

Semantics of hibana2077/torchwarp src/torchwarp/jeanie/functional.py:28-175
(Wang et al., IJCV 2024, Algorithm 1 and its two-axis extension): every
entry point takes a batch; shifts are clamped to K-1; a 4-D query/cost has one
viewpoint axis.  The DP, the (squared) Euclidean and rbf costs and their
backward passes run in the native library.
"""

import torch

from .. import _transforms
from . import _ops
from .distances import _native_cost, rbf_cost

_BACKENDS = ("auto", "cuda", "torch")
_METRICS = {"sqeuclidean": 0, "euclidean": 1}


def _feature_dtype(query, support):
    """The dtype the native kernels compute in for these features."""
    dtype = torch.promote_types(query.dtype, support.dtype)
    return dtype if dtype in (torch.float32, torch.float64) else torch.float32


def _check_common(gamma, max_shift_1, max_shift_2, backend):
    if gamma <= 0:
        raise ValueError("gamma must be > 0")
    if max_shift_1 < 0 or max_shift_2 < 0:
        raise ValueError("max shifts must be >= 0")
    if backend not in _BACKENDS:
        raise ValueError("backend must be one of {}".format(_BACKENDS))
    if backend == "torch":
        raise RuntimeError("torchwarp_b200 has no PyTorch (CPU) backend; use backend='auto' or "
                           "'cuda' with CUDA tensors")


def _jeanie_dp(cost, gamma=0.1, max_shift_1=1, max_shift_2=1, backend="auto",
               return_accumulator=False):
    """Batched JEANIE on a [B, K1, K2, T, U] cost tensor.

    Returns:
        (distance [B], accumulator [B, K1, K2, T, U] or None); the accumulator
        is differentiable.
    """
    if cost.ndim != 5:
        raise ValueError("cost must have shape [B, K1, K2, T, U]")
    if not cost.is_floating_point():
        raise TypeError("cost must be a floating-point tensor")
    _check_common(gamma, max_shift_1, max_shift_2, backend)
    B, K1, K2, T, U = cost.shape
    if min(K1, K2, T, U) == 0:
        raise ValueError("cost dimensions must be non-empty")
    if cost.dtype not in (torch.float32, torch.float64):
        cost = cost.float()
    s1 = min(int(max_shift_1), K1 - 1)
    s2 = min(int(max_shift_2), K2 - 1)
    if cost.dtype == torch.float32 and _ops.fused_supported(K1 * K2, T, U, 0, False, False):
        out, R, _ = _ops.fused_apply(None, None, cost, K1, K2, T, U, s1, s2, gamma, 0, False,
                                     return_accumulator)
        return out, (R if return_accumulator else None)
    out, R = _transforms.pick(_ops.JeanieDP, _ops.JeanieDPTraced).apply(
        cost, s1, s2, float(gamma), bool(return_accumulator))
    return out, (R if return_accumulator else None)


def _jeanie_dp_features(query, support, gamma=0.1, max_shift_1=1, max_shift_2=1,
                        metric="euclidean", backend="auto", return_accumulator=False):
    """Batched JEANIE straight from features: query [B, K1, K2, T, D], support [B, U, D]."""
    if query.ndim != 5 or support.ndim != 3:
        raise ValueError("query must be [B,K1,K2,T,D] and support [B,U,D]")
    if query.shape[0] != support.shape[0] or query.shape[-1] != support.shape[-1]:
        raise ValueError("query/support batch or feature dimensions do not match")
    if metric not in ("euclidean", "sqeuclidean", "rbf"):
        raise ValueError("metric must be 'euclidean', 'sqeuclidean' or 'rbf'")
    _check_common(gamma, max_shift_1, max_shift_2, backend)
    B, K1, K2, T, D = query.shape
    U = support.shape[1]
    if min(K1, K2, T, U) == 0:
        raise ValueError("query/support dimensions must be non-empty")
    if metric != "rbf" and _feature_dtype(query, support) == torch.float32 and \
            _ops.fused_supported(K1 * K2, T, U, D, False, True):
        # one native call per direction: cost, DP and chain rule on chip
        out, R, _ = _ops.fused_apply(
            query.to(torch.float32).reshape(B, K1 * K2 * T, D), support.to(torch.float32), None,
            K1, K2, T, U, min(int(max_shift_1), K1 - 1), min(int(max_shift_2), K2 - 1), gamma,
            _METRICS[metric], False, return_accumulator)
        return out, (R if return_accumulator else None)
    if metric == "rbf":
        cost = rbf_cost(query.reshape(B, K1 * K2, T, D), support).reshape(B, K1, K2, T, U)
    else:
        cost = _native_cost(query.reshape(B, K1 * K2, T, D), support,
                            _METRICS[metric]).reshape(B, K1, K2, T, U)
    return _jeanie_dp(cost, gamma, max_shift_1, max_shift_2, backend, return_accumulator)


def _max_shifts(max_shift, axes):
    """iota-max shift per viewpoint axis: an int applies to every axis."""
    if isinstance(max_shift, int):
        shifts = (max_shift,) * axes
    else:
        shifts = tuple(int(m) for m in max_shift)
        if len(shifts) != axes:
            raise ValueError("max_shift must be an int or a tuple of {} ints for {} viewpoint "
                             "axis/axes".format(axes, axes))
    if min(shifts) < 0:
        raise ValueError("max_shift must be >= 0")
    return shifts + (0,) * (2 - axes)


def jeanie(query, support, *, gamma=0.1, max_shift=1, metric="euclidean",
           return_accumulator=False, backend="auto"):
    """JEANIE between viewpoint-augmented queries and supports.

    Args:
        query: [B, K, T, D] (one viewpoint axis) or [B, K1, K2, T, D].
        support: [B, U, D] temporal blocks.
        gamma: SoftMin temperature (> 0).
        max_shift: iota-max shift; an int applies to every viewpoint axis.
        metric: "euclidean" (default), "sqeuclidean" or "rbf".
        return_accumulator: also return the differentiable DP tensor.
        backend: "auto" or "cuda".

    Returns:
        distance [B] (and the accumulator if requested).
    """
    if query.ndim not in (4, 5) or support.ndim != 3:
        raise ValueError("query must be [B,K,T,D] or [B,K1,K2,T,D] and support [B,U,D]")
    one_axis = query.ndim == 4
    s1, s2 = _max_shifts(max_shift, 1 if one_axis else 2)
    out, R = _jeanie_dp_features(query.unsqueeze(2) if one_axis else query, support, gamma,
                                 s1, s2, metric, backend, return_accumulator)
    if not return_accumulator:
        return out
    return out, (R[:, :, 0] if one_axis else R)


def jeanie_from_cost(cost, *, gamma=0.1, max_shift=1, return_accumulator=False, backend="auto"):
    """JEANIE on a precomputed cost [B, K, T, U] or [B, K1, K2, T, U].

    Returns:
        distance [B] (and the accumulator if requested).
    """
    if not cost.is_floating_point():
        raise TypeError("cost must be a floating-point tensor")
    if cost.ndim not in (4, 5):
        raise ValueError("cost must be [B,K,T,U] or [B,K1,K2,T,U]")
    one_axis = cost.ndim == 4
    s1, s2 = _max_shifts(max_shift, 1 if one_axis else 2)
    out, R = _jeanie_dp(cost.unsqueeze(2) if one_axis else cost, gamma, s1, s2, backend,
                        return_accumulator)
    if not return_accumulator:
        return out
    return out, (R[:, :, 0] if one_axis else R)
