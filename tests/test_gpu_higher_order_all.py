"""Higher-order derivatives of every path, against the official goldens (B200).

Mirrors the reference's parity tests for derivatives beyond the first order
(hibana2077/torchwarp tests/test_udtw_parity.py:53-125,
tests/test_jeanie_parity.py:91-222): MAML meta-gradients (create_graph), a
third derivative of uDTW with its penalty, gradgradcheck, and the torch.func
transforms (grad, jacrev, jacfwd, jvp, hessian = jacfwd(jacrev),
jacrev(jacrev)) of uDTW, JEANIE (with and without its accumulator), FVM and
soft-DTW.  First-order values come from the native kernels; higher orders go
through torch.func on the differentiable restatement of the recurrences.
Tolerances are the reference tests' (1e-9, 1e-7 for Hessians), in float64.
"""

import numpy as np
import pytest
import torch

import golden_data as G

pytestmark = pytest.mark.gpu

DEV = "cuda"
f64 = dict(dtype=torch.float64)
METHODS = ["gemm", "diff"]
SECOND_ORDER = ["jeanie_cost", "jeanie_features", "fvm", "soft_dtw"]


@pytest.fixture(scope="module")
def tw():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torchwarp_b200
    return torchwarp_b200


def _t(a):
    return torch.as_tensor(np.asarray(a), device=DEV, **f64)


def _close(a, b, tol=1e-9):
    torch.testing.assert_close(a.detach().cpu(), torch.as_tensor(np.asarray(b)), atol=tol,
                               rtol=tol)


def _scalar(module):
    def f(X, Y, SX, SY):
        d, p = module(X, Y, SX, SY)
        return d.sum() + 2.0 * p.sum()
    return f


# ---------------------------------------------------------------- uDTW

@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("normalize,bandwidth", [(False, None), (True, None), (False, 2)])
def test_udtw_maml(tw, method, normalize, bandwidth):
    ref = G.official("udtw.maml", normalize=normalize, bandwidth=bandwidth)
    X, Y, SX, SY = (_t(a) for a in ref["inputs"])
    w = _t(ref["W0"]).requires_grad_()
    f = _scalar(tw.UDTW(gamma=0.3, beta=0.8, normalize=normalize, bandwidth=bandwidth,
                        method=method))
    g, = torch.autograd.grad(f(X @ w.T, Y @ w.T, SX, SY), w, create_graph=True)
    w2 = w - 0.1 * g
    got = torch.autograd.grad(f(X @ w2.T, Y @ w2.T, SX, SY), w)[0]
    _close(got, ref["meta_grad"])


@pytest.mark.parametrize("method", METHODS)
def test_udtw_third_derivative(tw, method):
    ref = G.official("udtw.third_derivative")
    X, Y, SX, SY = (_t(a) for a in ref["inputs"])
    V = _t(ref["V"])
    f = _scalar(tw.UDTW(gamma=0.5, beta=0.8, method=method))
    t = torch.zeros((), device=DEV, **f64).requires_grad_()
    y = f(X + t * V, Y, SX, SY)
    for _ in range(3):
        y, = torch.autograd.grad(y, t, create_graph=True)
    _close(y, ref["d3"], tol=1e-7)


@pytest.mark.parametrize("method", METHODS)
def test_udtw_torch_func(tw, method):
    ref = G.official("udtw.func")
    X, Y, SX, SY = (_t(a) for a in ref["inputs"])
    m = tw.UDTW(gamma=0.4, beta=0.8, method=method)
    f = lambda x: _scalar(m)(x, Y, SX, SY)  # noqa: E731
    J = ref["jacobian"]
    _close(torch.func.grad(f)(X), J)
    _close(torch.func.jacrev(f)(X), J)
    _close(torch.func.jacfwd(f)(X), J)
    _, jvp = torch.func.jvp(f, (X,), (_t(ref["v"]),))
    _close(jvp, ref["jvp"])
    H = ref["hessian"]
    _close(torch.func.hessian(f)(X), H, tol=1e-7)
    _close(torch.func.jacrev(torch.func.jacrev(f))(X), H, tol=1e-7)


def test_udtw_gradgradcheck(tw):
    cost = torch.rand(2, 3, 4, device=DEV, **f64).requires_grad_()
    pen = torch.randn(2, 3, 4, device=DEV, **f64).requires_grad_()
    f = lambda c, p: tw.functional.udtw_from_cost(c, p, gamma=0.4)  # noqa: E731
    assert torch.autograd.gradgradcheck(f, (cost, pen))
    g = torch.Generator().manual_seed(0)
    ins = [torch.rand(1, 3, 2, generator=g, **f64), torch.rand(1, 4, 2, generator=g, **f64),
           0.5 + torch.rand(1, 3, 1, generator=g, **f64),
           0.5 + torch.rand(1, 4, 1, generator=g, **f64)]
    ins = [t.to(DEV).requires_grad_() for t in ins]
    h = lambda *a: tw.functional.udtw(*a, beta=0.7, gamma=0.4)  # noqa: E731
    assert torch.autograd.gradgradcheck(h, tuple(ins))


# --------------------------------------------------------- JEANIE / FVM

def _cost_loss(tw, cost, shift):
    d, R = tw.functional.jeanie_from_cost(cost[None], gamma=0.3, max_shift=shift,
                                          return_accumulator=True)
    return d[0] + 0.1 * (R ** 2).mean()


def _feat_loss(tw, q, s, metric, shift=1):
    d, R = tw.functional.jeanie(q[None], s[None], gamma=0.3, max_shift=shift, metric=metric,
                                return_accumulator=True)
    return d[0] + 0.1 * (R ** 2).mean()


@pytest.mark.parametrize("path", ["cost", "euclidean", "sqeuclidean"])
def test_jeanie_maml(tw, path):
    ref = G.official("parity.maml", path=path)

    def loss(qw, sw):
        if path == "cost":
            return _cost_loss(tw, tw.euclidean_cost(qw[None], sw[None])[0], 1)
        return _feat_loss(tw, qw, sw, path)

    w = _t(ref["W0"]).requires_grad_()
    a, b = _t(ref["q"]), _t(ref["s"])
    g, = torch.autograd.grad(loss(a @ w.T, b @ w.T), w, create_graph=True)
    w2 = w - 0.1 * g
    got = torch.autograd.grad(loss(a @ w2.T, b @ w2.T), w)[0]
    _close(got, ref["meta_grad"])


def _second_order_fn(tw, method, s):
    F = tw.functional
    if method == "jeanie_cost":
        return lambda x: F.jeanie_from_cost(x[None], gamma=0.3, max_shift=1)[0]
    if method == "jeanie_features":
        return lambda x: F.jeanie(x[None], s[None], gamma=0.3, max_shift=1)[0]
    if method == "fvm":
        return lambda x: F.fvm_from_cost(x[None], gamma=0.3)[0]
    return lambda x: F.soft_dtw_from_cost(x[None], gamma=0.3)[0]


@pytest.mark.parametrize("method", SECOND_ORDER)
def test_second_order_without_accumulator(tw, method):
    ref = G.official("parity.second_order", method=method)
    f = _second_order_fn(tw, method, _t(ref["s"]))
    x = _t(ref["x"])
    J = ref["jacobian"]
    _close(torch.func.grad(f)(x), J)
    _close(torch.func.jacrev(f)(x), J)
    _close(torch.func.jacfwd(f)(x), J)
    _, jvp = torch.func.jvp(f, (x,), (_t(ref["v"]),))
    _close(jvp, ref["jvp"])
    H = ref["hessian"]
    _close(torch.func.hessian(f)(x), H, tol=1e-7)
    _close(torch.func.jacrev(torch.func.jacrev(f))(x), H, tol=1e-7)
    _close(torch.autograd.functional.hessian(f, x), H, tol=1e-7)


@pytest.mark.parametrize("method", SECOND_ORDER)
def test_maml_without_accumulator(tw, method):
    ref = G.official("parity.maml_without_accumulator", method=method)
    F = tw.functional

    def loss(a, b):
        if method == "jeanie_cost":
            return F.jeanie_from_cost(tw.euclidean_cost(a[None], b[None]), gamma=0.3,
                                      max_shift=1)[0]
        if method == "jeanie_features":
            return F.jeanie(a[None], b[None], gamma=0.3, max_shift=1)[0]
        if method == "fvm":
            return F.fvm(a[None], b[None], gamma=0.3)[0]
        cost = ((a[:, None] - b[None]) ** 2).sum(-1)
        return F.soft_dtw_from_cost(cost[None], gamma=0.3)[0]

    w = _t(ref["W0"]).requires_grad_()
    a, b = _t(ref["q"]), _t(ref["s"])
    g, = torch.autograd.grad(loss(a @ w.T, b @ w.T), w, create_graph=True)
    w2 = w - 0.1 * g
    got = torch.autograd.grad(loss(a @ w2.T, b @ w2.T), w)[0]
    _close(got, ref["meta_grad"])


@pytest.mark.parametrize("path", ["cost", "euclidean"])
def test_jeanie_torch_func(tw, path):
    ref = G.official("parity.func", path=path)
    if path == "cost":
        f = lambda c: _cost_loss(tw, c, 1)  # noqa: E731
    else:
        s = _t(ref["s"])
        f = lambda qq: _feat_loss(tw, qq, s, path)  # noqa: E731
    x = _t(ref["x"])
    J = ref["jacobian"]
    _close(torch.func.grad(f)(x), J)
    _close(torch.func.jacrev(f)(x), J)
    _close(torch.func.jacfwd(f)(x), J)
    _, jvp = torch.func.jvp(f, (x,), (_t(ref["v"]),))
    _close(jvp, ref["jvp"])
    H = ref["hessian"]
    _close(torch.func.hessian(f)(x), H, tol=1e-7)
    _close(torch.func.jacrev(torch.func.jacrev(f))(x), H, tol=1e-7)


def test_jeanie_gradgradcheck(tw):
    F = tw.functional
    cost = torch.rand(2, 3, 3, 4, device=DEV, **f64).requires_grad_()
    assert torch.autograd.gradgradcheck(
        lambda c: F.jeanie_from_cost(c, gamma=0.5, max_shift=1), (cost,))
    assert torch.autograd.gradgradcheck(lambda c: F.fvm_from_cost(c, gamma=0.5), (cost,))
    assert torch.autograd.gradgradcheck(
        lambda c: F.soft_dtw_from_cost(c[:, 0], gamma=0.5), (cost,))
    q = torch.randn(1, 2, 3, 2, device=DEV, **f64).requires_grad_()
    s = torch.randn(1, 4, 2, device=DEV, **f64).requires_grad_()
    for metric in ("euclidean", "sqeuclidean", "rbf"):
        assert torch.autograd.gradgradcheck(
            lambda a, b: F.jeanie(a, b, gamma=0.5, max_shift=1, metric=metric), (q, s))
        assert torch.autograd.gradgradcheck(
            lambda a, b: F.fvm(a, b, gamma=0.5, metric=metric), (q, s))
    c5 = torch.rand(2, 2, 2, 3, 4, device=DEV, **f64).requires_grad_()
    assert torch.autograd.gradgradcheck(
        lambda c: tuple(F.jeanie_from_cost(c, gamma=0.5, max_shift=(1, 1),
                                           return_accumulator=True)), (c5,))


def test_fused_float32_second_order(tw):
    """float32 features take the fused kernels; their second derivatives go
    through the restatement and match the float64 ones to float32 accuracy."""
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 3, 5, 8, generator=g, **f64)
    s = torch.randn(2, 6, 8, generator=g, **f64)
    out = []
    for dt in (torch.float32, torch.float64):
        qq = q.to(dt).to(DEV).requires_grad_(True)
        ss = s.to(dt).to(DEV)
        d = tw.functional.jeanie(qq, ss, gamma=0.3, max_shift=1)
        gq, = torch.autograd.grad(d.sum(), qq, create_graph=True)
        h, = torch.autograd.grad((gq * gq).sum(), qq)
        out.append(h.double().cpu())
    err = (out[0] - out[1]).abs().max() / out[1].abs().max()
    assert err < 1e-3, err
