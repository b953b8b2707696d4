"""``nn.Module`` front ends for JEANIE and FVM (reference: src/torchwarp/jeanie/module.py)."""

import torch.nn as nn

from .functional import _max_shifts, jeanie
from .fvm import _METRICS, fvm


class JEANIE(nn.Module):
    """Joint tEmporal and cAmera viewpoiNt alIgnmEnt; see ``functional.jeanie``.

    Args:
        gamma: SoftMin temperature (> 0).
        max_shift: iota-max shift; an int applies to every viewpoint axis, a
            pair ``(azimuth, altitude)`` sets the two axes separately.
        metric: "euclidean" (default), "sqeuclidean" or "rbf".
        backend: "auto" or "cuda".
    """

    def __init__(self, gamma=0.1, max_shift=1, metric="euclidean", *, backend="auto"):
        super().__init__()
        if gamma <= 0:
            raise ValueError("gamma must be > 0")
        if metric not in _METRICS:
            raise ValueError("metric must be one of {}".format(tuple(_METRICS)))
        _max_shifts(max_shift, 1 if isinstance(max_shift, int) else len(max_shift))
        self.gamma = float(gamma)
        self.max_shift = max_shift if isinstance(max_shift, int) else tuple(max_shift)
        self.metric = metric
        self.backend = backend

    def forward(self, query, support, *, return_accumulator=False):
        return jeanie(query, support, gamma=self.gamma, max_shift=self.max_shift,
                      metric=self.metric, return_accumulator=return_accumulator,
                      backend=self.backend)

    def extra_repr(self):
        return "gamma={}, max_shift={}, metric={!r}, backend={!r}".format(
            self.gamma, self.max_shift, self.metric, self.backend)


class FVM(nn.Module):
    """Free Viewpoint Matching (JEANIE paper, Eq. 13); see ``functional.fvm``."""

    def __init__(self, gamma=0.1, metric="euclidean", *, backend="auto"):
        super().__init__()
        if gamma <= 0:
            raise ValueError("gamma must be > 0")
        if metric not in _METRICS:
            raise ValueError("metric must be one of {}".format(tuple(_METRICS)))
        self.gamma = float(gamma)
        self.metric = metric
        self.backend = backend

    def forward(self, query, support):
        return fvm(query, support, gamma=self.gamma, metric=self.metric, backend=self.backend)

    def extra_repr(self):
        return "gamma={}, metric={!r}, backend={!r}".format(self.gamma, self.metric, self.backend)
