"""torchwarp_b200: differentiable sequence alignment (soft-DTW, uDTW, JEANIE, FVM)
on NVIDIA B200 (sm_100a) kernels, with the public API of hibana2077/torchwarp.

    import torchwarp_b200 as torchwarp
    import torchwarp_b200.functional as TF
"""

from . import functional, paths
from .jeanie import FVM, JEANIE, euclidean_cost, rbf_cost, squared_euclidean_cost
from .sdtw import SoftDTW
from .udtw import UDTW

__version__ = "0.1.0"

__all__ = [
    "UDTW",
    "SoftDTW",
    "JEANIE",
    "FVM",
    "euclidean_cost",
    "squared_euclidean_cost",
    "rbf_cost",
    "functional",
    "paths",
]
