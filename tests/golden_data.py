"""Readers for the committed golden fixtures (tests/golden/*.npz).

``official(name, **params)`` returns one case of the reference's golden file
(outputs of the official uDTW / JEANIE code, float64) as a nested structure
of numpy arrays, keyed exactly like the reference's ``tests/golden.py``
(``key`` below follows its key format: the name, then ``|k=repr(v)`` for the
sorted parameters).  ``scaled(name)`` returns (inputs, kwargs, values,
grads) of a config-shaped case produced by the reference's PyTorch backend.
"""

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import inputs as _inputs  # noqa: E402

# Case lists used by the reference's golden generator (tests/golden.py:19-56
# of hibana2077/torchwarp); they name the stored cases.
UDTW_SHAPES = [(1, 1), (1, 6), (6, 1), (5, 8), (8, 5), (9, 9)]
GAMMAS = [0.01, 0.1, 1.0]
UDTW_BANDS = [(9, 9, 1), (9, 9, 2), (6, 10, 4), (10, 6, 4.5), (7, 7, 0)]
UDTW_BETAS = [0.0, 1.0, 3.0]
SDTW_SHAPES = [(1, 1), (1, 6), (6, 1), (5, 7), (8, 4), (9, 9)]
JEANIE_1D_SHAPES = [(1, 4, 5), (5, 6, 7), (5, 8, 5), (3, 1, 4)]
JEANIE_1D_SHIFTS = [0, 1, 2, 7]
JEANIE_2D_SHAPES = [(3, 3, 5, 6), (2, 4, 6, 4), (1, 3, 4, 4)]
JEANIE_2D_SHIFTS = [(0, 0), (1, 1), (1, 0), (2, 1)]
FVM_CASES = [("fvm_query_only_1d", (4, 5, 6)), ("fvm_query_only_2d", (3, 3, 5, 6)),
             ("fvm_1d_from_cost", (3, 4, 6, 5)), ("fvm_2d_from_cost", (2, 2, 3, 2, 5, 6))]
DISTANCES = ["euclidean_cost", "squared_euclidean_cost", "rbf_cost"]
METRICS = ["euclidean", "sqeuclidean", "rbf"]
FEATURES_1D = [(5, 6, 8, 1), (3, 9, 4, 2), (1, 5, 5, 0)]
ACCUMULATOR_COST = [(4, 5, 7, 1), (3, 7, 4, 2), (1, 4, 4, 0)]
UDTW_LARGE = [(2, 40, 50)]
LARGE_COST = [("soft_dtw", (60, 70), None), ("jeanie_1d_from_cost", (5, 30, 40), 2),
              ("jeanie_1d_from_cost", (4, 35, 20), 1), ("jeanie_2d_from_cost", (3, 3, 20, 25), (1, 1)),
              ("fvm_query_only_1d", (5, 40, 50), None), ("fvm_query_only_2d", (2, 3, 30, 35), None)]

_OFFICIAL = None
_SCALED = None


def key(name, /, **params):
    return name + "".join("|{}={!r}".format(k, params[k]) for k in sorted(params))


def _unflatten(data, prefix):
    if prefix in data:
        return data[prefix]
    if prefix + "::len" in data:
        return [_unflatten(data, "{}::{}".format(prefix, i))
                for i in range(int(data[prefix + "::len"]))]
    fields = {}
    head = prefix + "::"
    for k in data:
        if k.startswith(head):
            f = k[len(head):].split("::")[0]
            if f not in fields:
                fields[f] = _unflatten(data, head + f)
    if not fields:
        raise KeyError(prefix)
    return fields


def official(name, /, **params):
    global _OFFICIAL
    if _OFFICIAL is None:
        with np.load(HERE / "golden" / "official.npz") as z:
            _OFFICIAL = dict(z.items())
    return _unflatten(_OFFICIAL, key(name, **params))


def scaled(name):
    """(inputs as float64 numpy, kwargs, values, grads) of a scaled case."""
    global _SCALED
    if _SCALED is None:
        with np.load(HERE / "golden" / "scaled.npz") as z:
            _SCALED = dict(z.items())
    tensors, kwargs = _inputs.make(name)
    ins = [t.numpy() for t, _ in tensors]
    vals = [_SCALED["{}::value::{}".format(name, i)] for i in range(2)
            if "{}::value::{}".format(name, i) in _SCALED]
    grads = [_SCALED["{}::grad::{}".format(name, i)] for i in range(4)
             if "{}::grad::{}".format(name, i) in _SCALED]
    return ins, kwargs, vals, grads


SCALED_CASES = list(_inputs.SCALED_CASES)


_HIGHER = None
HIGHER_COST_CASES = ["c7x9", "c33x40", "c70x65", "c64x130", "c40x44_band6", "c20x20_g005"]
HIGHER_FEAT_CASES = ["f20x24d5", "f70x66d8"]


def higher(name):
    """{field: array} of a higher-order case (tests/golden/make_higher_order.py)."""
    global _HIGHER
    if _HIGHER is None:
        with np.load(HERE / "golden" / "higher_order.npz") as z:
            _HIGHER = dict(z.items())
    head = name + "/"
    return {k[len(head):]: v for k, v in _HIGHER.items() if k.startswith(head)}
