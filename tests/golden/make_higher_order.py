"""Write tests/golden/higher_order.npz: second-order and forward-mode derivatives
of soft-DTW from the reference's own autograd DP (run in a container that has
the reference).

The reference differentiates through its first-order backward with a
pure-PyTorch anti-diagonal DP (``torchwarp/udtw/_autograd.py`` of
hibana2077/torchwarp, routed at ``udtw/_ops.py:226-258``).  This script runs
that module in float64 on the CPU and records, per case:

* cost cases (soft-DTW on a cost C, per-pair seeds g, direction V, tangent T):
  ``d``; ``dC`` = d(sum g d)/dC; ``hvp_C``, ``hvp_g`` = the gradients of
  <V, dC> with respect to C and g (double backward); ``jvp`` = the forward-mode
  derivative of d along T.
* feature cases (soft-DTW on features X, Y with the squared-Euclidean cost):
  ``d``, ``dX``, ``dY`` and the gradients of <VX, dX> + <VY, dY> with respect to
  X, Y and g.

Usage (needs the reference importable, e.g. PYTHONPATH=<reference>/src):

    python tests/golden/make_higher_order.py

Only this script touches the reference; the tests read the .npz.
"""

from pathlib import Path

import numpy as np
import torch
from torchwarp.udtw import _autograd as A

OUT = Path(__file__).resolve().parent / "higher_order.npz"

COST_CASES = {  # name: (B, N, M, gamma, bandwidth)
    "c7x9": (2, 7, 9, 0.3, 0),
    "c33x40": (2, 33, 40, 0.3, 0),
    "c70x65": (2, 70, 65, 0.5, 0),
    "c64x130": (2, 64, 130, 0.3, 0),     # N a multiple of the band height
    "c40x44_band6": (2, 40, 44, 0.3, 6),
    "c20x20_g005": (3, 20, 20, 0.05, 0),
}
FEAT_CASES = {  # name: (B, N, M, D, gamma)
    "f20x24d5": (2, 20, 24, 5, 0.3),
    "f70x66d8": (2, 70, 66, 8, 0.5),
}


def sdtw_cost(C, gamma, band):
    return A.udtw(C, torch.zeros_like(C), gamma, band)[0]


def sqeuclid(X, Y):
    ones_x = X.new_ones(X.shape[:2])
    ones_y = Y.new_ones(Y.shape[:2])
    return A.matrices_from_features(X, Y, ones_x, ones_y, 0.0, 1e-6)[0]


def main():
    g = torch.Generator().manual_seed(2024)
    out = {}
    for name, (B, N, M, gamma, band) in COST_CASES.items():
        C = torch.rand(B, N, M, generator=g, dtype=torch.float64)
        V = torch.randn(B, N, M, generator=g, dtype=torch.float64)
        T = torch.randn(B, N, M, generator=g, dtype=torch.float64)
        w = torch.rand(B, generator=g, dtype=torch.float64) + 0.5
        c = C.clone().requires_grad_(True)
        wg = w.clone().requires_grad_(True)
        d = sdtw_cost(c, gamma, band)
        (dC,) = torch.autograd.grad((d * wg).sum(), c, create_graph=True)
        hC, hg = torch.autograd.grad((dC * V).sum(), (c, wg))
        jvp = torch.func.jvp(lambda x: sdtw_cost(x, gamma, band), (C,), (T,))[1]
        for k, v in dict(C=C, V=V, T=T, g=w, d=d.detach(), dC=dC.detach(), hvp_C=hC, hvp_g=hg,
                         jvp=jvp).items():
            out["{}/{}".format(name, k)] = v.numpy()
        out["{}/args".format(name)] = np.array([gamma, band], dtype=np.float64)
    for name, (B, N, M, D, gamma) in FEAT_CASES.items():
        X = torch.randn(B, N, D, generator=g, dtype=torch.float64)
        Y = torch.randn(B, M, D, generator=g, dtype=torch.float64)
        VX = torch.randn(B, N, D, generator=g, dtype=torch.float64)
        VY = torch.randn(B, M, D, generator=g, dtype=torch.float64)
        w = torch.rand(B, generator=g, dtype=torch.float64) + 0.5
        x, y = X.clone().requires_grad_(True), Y.clone().requires_grad_(True)
        wg = w.clone().requires_grad_(True)
        d = sdtw_cost(sqeuclid(x, y), gamma, 0)
        dX, dY = torch.autograd.grad((d * wg).sum(), (x, y), create_graph=True)
        hX, hY, hg = torch.autograd.grad((dX * VX).sum() + (dY * VY).sum(), (x, y, wg))
        for k, v in dict(X=X, Y=Y, VX=VX, VY=VY, g=w, d=d.detach(), dX=dX.detach(),
                         dY=dY.detach(), hvp_X=hX, hvp_Y=hY, hvp_g=hg).items():
            out["{}/{}".format(name, k)] = v.numpy()
        out["{}/args".format(name)] = np.array([gamma], dtype=np.float64)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, len(out), "arrays")


if __name__ == "__main__":
    main()
