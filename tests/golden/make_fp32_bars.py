"""Float32 accuracy bars of the reference, per benchmark configuration.

The reference's own float32 does not meet a fixed gradient tolerance
against its float64 at small gamma and long sequences (its documentation
says so, and this script measures it).  So the float32 parity of this
package is judged per configuration against the reference's float32 error:
this script runs the reference's PyTorch backend (``backend="torch"`` on
CPU) in float64 and in float32 on the same seeded inputs
(``inputs.CONFIG_CASES``) and writes ``fp32_bars.npz`` with, per case:

* ``<case>::value64``       the reference's float64 forward values [B];
* ``<case>::gsum64::<i>``   sum, sum of squares and max |.| of the float64
                            gradient of input i (a checksum of the truth);
* ``<case>::gsub64::<i>``   about 2000 evenly spaced elements of that
                            gradient (flattened, stride ``gstride``);
* ``<case>::gstride::<i>``  that stride;
* ``<case>::fwd_rel``       max |d32 - d64| / |d64| of the reference float32;
* ``<case>::maxnorm::<i>``  max |g32 - g64| / max |g64| for input i;
* ``<case>::fail::<i>``     fraction of elements of input i's gradient with
                            |g32 - g64| > 1e-6 + 1e-4 |g64|.

Usage (needs the reference importable):

    python tests/golden/make_fp32_bars.py <reference_root>

The tests read only the .npz file.
"""

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import inputs as I  # noqa: E402


def error_metrics(v32, v64, g32, g64):
    """(fwd_rel, [maxnorm per gradient], [fail fraction per gradient])."""
    v32, v64 = np.asarray(v32, np.float64), np.asarray(v64, np.float64)
    fwd = float(np.max(np.abs(v32 - v64) / np.abs(v64))) if v64.size else 0.0
    mn, fail = [], []
    for a, b in zip(g32, g64):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        err = np.abs(a - b)
        mn.append(float(err.max() / max(np.abs(b).max(), 1e-300)))
        fail.append(float(np.mean(err > 1e-6 + 1e-4 * np.abs(b))))
    return fwd, mn, fail


def run(F, name, dtype):
    build, _, wrt = I.CONFIG_CASES[name]
    tensors, kw = build()
    xs = [t.to(dtype).requires_grad_(k in wrt) for k, t in enumerate(tensors)]
    d, loss = I.config_loss(F, name, xs, kw, backend="torch")
    grads = torch.autograd.grad(loss, [xs[k] for k in wrt])
    return d.detach().double().numpy(), [g.double().numpy() for g in grads]


def main(root):
    sys.path.insert(0, str(Path(root) / "src"))
    import torchwarp.functional as F  # the reference package

    torch.set_num_threads(max(1, torch.get_num_threads()))
    out = {}
    for name in I.CONFIG_CASES:
        v64, g64 = run(F, name, torch.float64)
        v32, g32 = run(F, name, torch.float32)
        fwd, mn, fail = error_metrics(v32, v64, g32, g64)
        out[name + "::value64"] = v64
        out[name + "::fwd_rel"] = np.array(fwd)
        for i, g in enumerate(g64):
            out["{}::gsum64::{}".format(name, i)] = np.array(
                [g.sum(), (g * g).sum(), np.abs(g).max()])
            stride = max(1, g.size // 2000) | 1
            out["{}::gstride::{}".format(name, i)] = np.array(stride)
            out["{}::gsub64::{}".format(name, i)] = g.reshape(-1)[::stride].copy()
            out["{}::maxnorm::{}".format(name, i)] = np.array(mn[i])
            out["{}::fail::{}".format(name, i)] = np.array(fail[i])
        print("{:20s} fwd_rel {:.2e}  maxnorm {}  fail {}".format(
            name, fwd, " ".join("%.2e" % m for m in mn), " ".join("%.3f" % f for f in fail)))
    np.savez_compressed(HERE / "fp32_bars.npz", **out)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_fp32_bars.py <reference_root>")
    main(sys.argv[1])
