"""torch.func.vmap, per-sample gradients, jacrev, torch.compile(fullgraph=True)
and autocast through the native operators (B200).

Mirrors the transform tests of the reference (hibana2077/torchwarp
tests/test_udtw_parity.py:126-173 and tests/test_jeanie_parity.py:224-279):
vmapped calls must reproduce the official golden values ``udtw.vmap`` and
``parity.vmap``; per-sample gradients (vmap of grad) must equal the full
batch gradient; compiled functions must give the eager values and
gradients; autocast runs the DP and the fused costs in float32.
"""

import numpy as np
import pytest
import torch

import golden_data as G

pytestmark = pytest.mark.gpu

DEV = "cuda"
f64 = dict(dtype=torch.float64)


@pytest.fixture(scope="module")
def tw():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torchwarp_b200
    return torchwarp_b200


def _t(a):
    return torch.as_tensor(np.asarray(a), device=DEV, **f64)


def _close(a, b, tol=1e-9):
    torch.testing.assert_close(a, b, atol=tol, rtol=tol)


def _scalar(module):
    def f(X, Y, SX, SY):
        d, p = module(X, Y, SX, SY)
        return d.sum() + 2.0 * p.sum()
    return f


def _udtw_inputs(B=2, N=5, M=6, D=4, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [t.to(DEV) for t in (torch.rand(B, N, D, generator=g, **f64),
                                torch.rand(B, M, D, generator=g, **f64),
                                0.5 + torch.rand(B, N, 1, generator=g, **f64),
                                0.5 + torch.rand(B, M, 1, generator=g, **f64))]


@pytest.mark.parametrize("method", ["gemm", "diff"])
def test_udtw_vmap_golden(tw, method):
    ref = G.official("udtw.vmap")
    X, Y, SX, SY = (_t(a) for a in ref["inputs"])
    stack = lambda t: torch.stack([t, 1.1 * t, 0.9 * t])  # noqa: E731
    m = tw.UDTW(gamma=0.3, beta=0.5, method=method)
    d, p = torch.func.vmap(m)(stack(X), stack(Y), stack(SX), stack(SY))
    _close(d.cpu(), torch.as_tensor(ref["distance"]))
    _close(p.cpu(), torch.as_tensor(ref["penalty"]))
    # per-sample gradients: vmap(grad) against the batch gradient
    g = torch.func.vmap(torch.func.grad(
        lambda x, y, sx, sy: _scalar(m)(x[None], y[None], sx[None], sy[None]),
        argnums=(0, 1, 2, 3)))
    per = g(X, Y, SX, SY)
    full = torch.func.grad(_scalar(m), argnums=(0, 1, 2, 3))(X, Y, SX, SY)
    for a, b in zip(per, full):
        _close(a, b)


def test_soft_dtw_vmap_and_jacrev(tw):
    g = torch.Generator().manual_seed(3)
    X = torch.randn(4, 3, 9, 5, generator=g, **f64).to(DEV)
    Y = torch.randn(4, 3, 11, 5, generator=g, **f64).to(DEV)
    f = lambda x, y: tw.functional.soft_dtw(x, y, gamma=0.2)  # noqa: E731
    got = torch.func.vmap(f)(X, Y)
    want = f(X.reshape(12, 9, 5), Y.reshape(12, 11, 5)).reshape(4, 3)
    _close(got, want)
    # per-sample gradients of a vmapped batch
    per = torch.func.vmap(torch.func.grad(lambda x, y: f(x, y).sum()))(X, Y)
    x = X.reshape(12, 9, 5).clone().requires_grad_(True)
    f(x, Y.reshape(12, 11, 5)).sum().backward()
    _close(per, x.grad.reshape(4, 3, 9, 5))
    # jacrev: vmapped cotangents of an unbatched forward
    J = torch.func.jacrev(f)(X[0], Y[0])                      # [3, 3, 9, 5]
    for b in range(3):
        _close(J[b, b], x.grad[b])
        assert torch.count_nonzero(J[b, [k for k in range(3) if k != b]]) == 0


def test_soft_dtw_from_cost_vmap(tw):
    g = torch.Generator().manual_seed(4)
    C = torch.rand(3, 2, 17, 13, generator=g, **f64).to(DEV)
    f = lambda c: tw.functional.soft_dtw_from_cost(c, gamma=0.1)  # noqa: E731
    _close(torch.func.vmap(f)(C), f(C.reshape(6, 17, 13)).reshape(3, 2))
    per = torch.func.vmap(torch.func.grad(lambda c: f(c).sum()))(C)
    c = C.reshape(6, 17, 13).clone().requires_grad_(True)
    f(c).sum().backward()
    _close(per, c.grad.reshape(3, 2, 17, 13))


def test_udtw_from_cost_vmap(tw):
    g = torch.Generator().manual_seed(5)
    C = torch.rand(2, 3, 12, 15, generator=g, **f64).to(DEV)
    P = torch.rand(2, 3, 12, 15, generator=g, **f64).to(DEV)
    f = lambda c, p: tw.functional.udtw_from_cost(c, p, gamma=0.3)  # noqa: E731
    d, p = torch.func.vmap(f)(C, P)
    dw, pw = f(C.reshape(6, 12, 15), P.reshape(6, 12, 15))
    _close(d, dw.reshape(2, 3))
    _close(p, pw.reshape(2, 3))
    per = torch.func.vmap(torch.func.grad(lambda c, p: sum(v.sum() for v in f(c, p)),
                                          argnums=(0, 1)))(C, P)
    c = C.reshape(6, 12, 15).clone().requires_grad_(True)
    q = P.reshape(6, 12, 15).clone().requires_grad_(True)
    sum(v.sum() for v in f(c, q)).backward()
    _close(per[0], c.grad.reshape(C.shape))
    _close(per[1], q.grad.reshape(P.shape))


def test_jeanie_vmap_golden(tw):
    ref = G.official("parity.vmap")
    TF = tw.functional
    got = torch.func.vmap(lambda c: TF.jeanie_from_cost(c, gamma=0.3, max_shift=1))(
        _t(ref["cost"]))
    _close(got.cpu(), torch.as_tensor(ref["cost_value"]))
    q, s = _t(ref["q"]), _t(ref["s"])
    got = torch.func.vmap(lambda a, b: TF.jeanie(a, b, gamma=0.3, max_shift=1))(q, s)
    _close(got.cpu(), torch.as_tensor(ref["features_value"]))
    f = lambda a, b: TF.jeanie(a, b, gamma=0.3, max_shift=1)  # noqa: E731
    per = torch.func.vmap(torch.func.grad(lambda a, b: f(a[None], b[None])[0]))(q[0], s[0])
    full = torch.func.grad(lambda a, b: f(a, b).sum())(q[0], s[0])
    _close(per, full)


def test_fvm_vmap(tw):
    g = torch.Generator().manual_seed(6)
    q = torch.randn(2, 3, 4, 6, 5, generator=g, **f64).to(DEV)
    s = torch.randn(2, 3, 7, 5, generator=g, **f64).to(DEV)
    f = lambda a, b: tw.functional.fvm(a, b, gamma=0.2)  # noqa: E731
    _close(torch.func.vmap(f)(q, s), f(q.reshape(6, 4, 6, 5), s.reshape(6, 7, 5)).reshape(2, 3))


@pytest.mark.parametrize("method", ["gemm", "diff"])
def test_udtw_compile_fullgraph(tw, method):
    torch._dynamo.reset()
    X, Y, SX, SY = (t.requires_grad_() for t in _udtw_inputs(B=3, N=5, M=7))
    m = tw.UDTW(gamma=0.3, beta=0.8, normalize=True, method=method)
    f = _scalar(m)
    compiled = torch.compile(f, fullgraph=True)
    want = f(X, Y, SX, SY)
    got = compiled(X, Y, SX, SY)
    _close(got, want)
    for a, b in zip(torch.autograd.grad(got, (X, Y, SX, SY)),
                    torch.autograd.grad(want, (X, Y, SX, SY))):
        _close(a, b)


def test_soft_dtw_compile_fullgraph(tw):
    torch._dynamo.reset()
    g = torch.Generator().manual_seed(7)
    X = torch.randn(3, 40, 64, generator=g).to(DEV).requires_grad_()
    Y = torch.randn(3, 48, 64, generator=g).to(DEV).requires_grad_()
    f = lambda x, y: tw.functional.soft_dtw(x, y, gamma=0.1).sum()  # noqa: E731
    compiled = torch.compile(f, fullgraph=True)
    want, got = f(X, Y), compiled(X, Y)
    torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-5)
    for a, b in zip(torch.autograd.grad(got, (X, Y)), torch.autograd.grad(want, (X, Y))):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("path", ["cost", "euclidean"])
def test_jeanie_compile_fullgraph(tw, path):
    torch._dynamo.reset()
    TF = tw.functional
    q = torch.randn(2, 3, 5, 4, device=DEV, **f64).requires_grad_()
    s = torch.randn(2, 6, 4, device=DEV, **f64).requires_grad_()
    if path == "cost":
        def f(q, s):
            d, R = TF.jeanie_from_cost(tw.euclidean_cost(q, s), gamma=0.3, max_shift=1,
                                       return_accumulator=True)
            return d.sum() + 0.1 * (R ** 2).mean()
    else:
        def f(q, s):
            d, R = TF.jeanie(q, s, gamma=0.3, max_shift=1, return_accumulator=True)
            return d.sum() + 0.1 * (R ** 2).mean()
    compiled = torch.compile(f, fullgraph=True)
    want, got = f(q, s), compiled(q, s)
    _close(got, want)
    for a, b in zip(torch.autograd.grad(got, (q, s)), torch.autograd.grad(want, (q, s))):
        _close(a, b)


def test_udtw_autocast_runs_in_float32(tw):
    X, Y, SX, SY = (t.float().requires_grad_() for t in _udtw_inputs(B=2, N=5, M=6))
    lin = torch.nn.Linear(4, 4).to(DEV)
    for method in ("gemm", "diff"):
        m = tw.UDTW(gamma=0.3, method=method)
        with torch.autocast("cuda", dtype=torch.float16):
            d, p = m(lin(X), lin(Y), SX, SY)
        assert d.dtype == torch.float32 and p.dtype == torch.float32
        (d.sum() + p.sum()).backward()
        assert torch.isfinite(X.grad).all()
        ref_d, _ = m(lin(X).float(), lin(Y).float(), SX, SY)
        torch.testing.assert_close(d, ref_d, atol=5e-2, rtol=5e-3)
        X.grad = None


def test_jeanie_autocast_runs_in_float32(tw):
    TF = tw.functional
    q = torch.randn(2, 3, 5, 8, device=DEV).requires_grad_()
    s = torch.randn(2, 6, 8, device=DEV)
    lin = torch.nn.Linear(8, 8).to(DEV)
    with torch.autocast("cuda", dtype=torch.float16):
        a = TF.jeanie(lin(q), lin(s), gamma=0.3, max_shift=1)
        b = TF.jeanie_from_cost(tw.euclidean_cost(lin(q), lin(s)), gamma=0.3, max_shift=1)
    assert a.dtype == torch.float32 and b.dtype == torch.float32
    (a.sum() + b.sum()).backward()
    assert torch.isfinite(q.grad).all()
