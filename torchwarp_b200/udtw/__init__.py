"""Uncertainty-DTW (ECCV 2022)."""

from .functional import UDTWOutput, pairwise_matrices, udtw, udtw_from_cost
from .module import UDTW

__all__ = ["UDTW", "udtw", "udtw_from_cost", "pairwise_matrices", "UDTWOutput"]
