"""Second-order and forward-mode derivatives of soft-DTW through the native
kernels (B200), against the reference's own autograd DP.

The fixtures (tests/golden/make_higher_order.py) are float64 outputs of the
reference's pure-PyTorch DP (``torchwarp/udtw/_autograd.py`` of
hibana2077/torchwarp), which is how the reference differentiates through its
first-order backward.  Here the same quantities come from native kernels:
the double backward is a Hessian-vector product run as the uDTW forward and
backward with the direction as the penalty, and jvp is the uDTW forward with
the tangent as the penalty.
"""

import numpy as np
import pytest
import torch

import golden_data as G

pytestmark = pytest.mark.gpu

DEV = "cuda"
ATOL, RTOL = 1e-9, 1e-8   # float64; second derivatives take more arithmetic than values


@pytest.fixture(scope="module")
def tw():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torchwarp_b200
    return torchwarp_b200


def _t(a, dtype=torch.float64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def _close(got, want, atol=ATOL, rtol=RTOL):
    np.testing.assert_allclose(got.detach().double().cpu().numpy(), np.asarray(want), atol=atol,
                               rtol=rtol)


def _cost_second_order(tw, h, dtype=torch.float64):
    gamma, band = h["args"]
    c = _t(h["C"], dtype).requires_grad_(True)
    g = _t(h["g"], dtype).requires_grad_(True)
    d = tw.functional.soft_dtw_from_cost(c, gamma=float(gamma), bandwidth=float(band) or None)
    (dC,) = torch.autograd.grad((d * g).sum(), c, create_graph=True)
    hC, hg = torch.autograd.grad((dC * _t(h["V"], dtype)).sum(), (c, g))
    return d, dC, hC, hg


@pytest.mark.parametrize("name", G.HIGHER_COST_CASES)
def test_cost_double_backward(tw, name):
    h = G.higher(name)
    d, dC, hC, hg = _cost_second_order(tw, h)
    _close(d, h["d"], 1e-10, 1e-9)
    _close(dC, h["dC"], 1e-10, 1e-9)
    _close(hC, h["hvp_C"])
    _close(hg, h["hvp_g"])
    assert tw._native.lib().tw_device_error() == 0


@pytest.mark.parametrize("name", G.HIGHER_COST_CASES)
def test_cost_jvp(tw, name):
    h = G.higher(name)
    gamma, band = h["args"]
    f = lambda c: tw.functional.soft_dtw_from_cost(c, gamma=float(gamma),  # noqa: E731
                                                   bandwidth=float(band) or None)
    d, jvp = torch.func.jvp(f, (_t(h["C"]),), (_t(h["T"]),))
    _close(d, h["d"], 1e-10, 1e-9)
    _close(jvp, h["jvp"])


@pytest.mark.parametrize("name", G.HIGHER_FEAT_CASES)
def test_features_double_backward(tw, name):
    h = G.higher(name)
    (gamma,) = h["args"]
    x = _t(h["X"]).requires_grad_(True)
    y = _t(h["Y"]).requires_grad_(True)
    g = _t(h["g"]).requires_grad_(True)
    d = tw.functional.soft_dtw(x, y, gamma=float(gamma))
    dX, dY = torch.autograd.grad((d * g).sum(), (x, y), create_graph=True)
    hX, hY, hg = torch.autograd.grad((dX * _t(h["VX"])).sum() + (dY * _t(h["VY"])).sum(),
                                     (x, y, g))
    _close(d, h["d"], 1e-10, 1e-9)
    _close(dX, h["dX"], 1e-9, 1e-8)
    _close(dY, h["dY"], 1e-9, 1e-8)
    _close(hX, h["hvp_X"], 1e-8, 1e-7)
    _close(hY, h["hvp_Y"], 1e-8, 1e-7)
    _close(hg, h["hvp_g"], 1e-8, 1e-7)


def test_features_jvp_matches_cost_path(tw):
    """jvp on features equals the jvp of the cost path along the cost's tangent."""
    h = G.higher("f20x24d5")
    (gamma,) = h["args"]
    X, Y, VX, VY = (_t(h[k]) for k in ("X", "Y", "VX", "VY"))
    f = lambda a, b: tw.functional.soft_dtw(a, b, gamma=float(gamma))  # noqa: E731
    d, jvp = torch.func.jvp(f, (X, Y), (VX, VY))
    eps = 1e-6
    fd = (f(X + eps * VX, Y + eps * VY) - f(X - eps * VX, Y - eps * VY)) / (2 * eps)
    _close(d, h["d"], 1e-10, 1e-9)
    _close(jvp, fd.cpu().numpy(), 1e-6, 1e-6)


def test_udtw_jvp_against_central_difference(tw):
    """jvp of uDTW on matrices (distance and penalty sum) along tangents of
    both, against a float64 central difference."""
    g = torch.Generator().manual_seed(3)
    B, N, M = 3, 45, 52
    C = torch.rand(B, N, M, generator=g, dtype=torch.float64).to(DEV)
    Q = torch.randn(B, N, M, generator=g, dtype=torch.float64).to(DEV)
    Ct = torch.randn(B, N, M, generator=g, dtype=torch.float64).to(DEV)
    Qt = torch.randn(B, N, M, generator=g, dtype=torch.float64).to(DEV)
    f = lambda c, q: tw.functional.udtw_from_cost(c, q, gamma=0.3)  # noqa: E731
    (d, p), (d_t, p_t) = torch.func.jvp(f, (C, Q), (Ct, Qt))
    eps = 1e-6
    dp_, pp_ = f(C + eps * Ct, Q + eps * Qt)
    dm_, pm_ = f(C - eps * Ct, Q - eps * Qt)
    _close(d_t, ((dp_ - dm_) / (2 * eps)).cpu().numpy(), 1e-6, 1e-6)
    _close(p_t, ((pp_ - pm_) / (2 * eps)).cpu().numpy(), 1e-6, 1e-6)


def test_cost_double_backward_fp32(tw):
    """float32 double backward against the float64 fixture: max-normalised
    error within the reference's float32 bar (1e-3)."""
    h = G.higher("c70x65")
    _, _, hC, hg = _cost_second_order(tw, h, torch.float32)
    for got, want in ((hC, h["hvp_C"]), (hg, h["hvp_g"])):
        err = np.abs(got.detach().double().cpu().numpy() - want).max() / np.abs(want).max()
        assert err < 1e-3, err


def _third_fd(tw, f, c, V, eps=1e-6):
    """d/de of <H(c + e V) V, V> by a central difference of the second
    derivative, and the third derivative from autograd."""
    def second(x):
        x = x.detach().requires_grad_(True)
        (g,) = torch.autograd.grad(f(x), x, create_graph=True)
        (h,) = torch.autograd.grad((g * V).sum(), x, create_graph=True)
        return h, x
    h, x = second(c)
    (t3,) = torch.autograd.grad((h * V).sum(), x)
    hp, _ = second(c + eps * V)
    hm, _ = second(c - eps * V)
    fd = (((hp - hm) * V).sum() / (2 * eps)).item()
    return (t3 * V).sum().item(), fd


def test_soft_dtw_third_order(tw):
    """Third derivatives of soft-DTW (through the restatement) against a
    central difference of the native second derivative."""
    h = G.higher("c7x9")
    c = _t(h["C"])
    V = _t(h["V"])
    got, fd = _third_fd(tw, lambda x: tw.functional.soft_dtw_from_cost(x, gamma=0.3).sum(), c,
                        V)
    assert abs(got - fd) <= 1e-5 * max(1.0, abs(fd)), (got, fd)


def test_udtw_second_order(tw, orc):
    """Second derivatives of uDTW with a penalty: the Hessian-vector product
    along (V_C, V_Q) against a central difference of the native gradient."""
    g = torch.Generator().manual_seed(4)
    C = torch.rand(2, 9, 11, generator=g, dtype=torch.float64).to(DEV)
    Q = torch.randn(2, 9, 11, generator=g, dtype=torch.float64).to(DEV)
    VC = torch.randn(2, 9, 11, generator=g, dtype=torch.float64).to(DEV)
    VQ = torch.randn(2, 9, 11, generator=g, dtype=torch.float64).to(DEV)

    def grads(c, q, create):
        c, q = c.detach().requires_grad_(True), q.detach().requires_grad_(True)
        d, p = tw.functional.udtw_from_cost(c, q, gamma=0.3)
        return torch.autograd.grad((d + 2.0 * p).sum(), (c, q), create_graph=create), (c, q)

    (gc, gq), (c, q) = grads(C, Q, True)
    hc, hq = torch.autograd.grad((gc * VC).sum() + (gq * VQ).sum(), (c, q))
    eps = 1e-6
    (pc, pq), _ = grads(C + eps * VC, Q + eps * VQ, False)
    (mc, mq), _ = grads(C - eps * VC, Q - eps * VQ, False)
    for got, fd in ((hc, (pc - mc) / (2 * eps)), (hq, (pq - mq) / (2 * eps))):
        _close(got, fd.cpu().numpy(), 1e-6, 1e-6)


def _fd_check(f, primals, tangents, eps=1e-6):
    """torch.func.jvp against a float64 central difference."""
    _, jvp = torch.func.jvp(f, primals, tangents)
    plus = f(*[p + eps * t for p, t in zip(primals, tangents)])
    minus = f(*[p - eps * t for p, t in zip(primals, tangents)])
    _close(jvp, ((plus - minus) / (2 * eps)).cpu().numpy(), 1e-6, 1e-6)


def _rn(g, *shape):
    return torch.randn(*shape, generator=g, dtype=torch.float64).to(DEV)


@pytest.mark.parametrize("case", ["jeanie_cost", "jeanie_euclidean", "jeanie_sqeuclidean",
                                  "fvm_cost", "fvm_features", "fvm_support_viewpoints"])
def test_jeanie_fvm_jvp(tw, case):
    """Forward mode of JEANIE and FVM: native backward weights (JEANIE DP,
    FVM soft-min), the cost's tangent and the soft-DTW jvp, against central
    differences."""
    g = torch.Generator().manual_seed(len(case))
    TF = tw.functional
    if case == "jeanie_cost":
        c = torch.rand(2, 3, 2, 6, 7, generator=g, dtype=torch.float64).to(DEV)
        _fd_check(lambda x: TF.jeanie_from_cost(x, gamma=0.1, max_shift=1), (c,), (_rn(g, *c.shape),))
    elif case.startswith("jeanie_"):
        metric = case.split("_")[1]
        q, s = _rn(g, 2, 3, 2, 6, 5), _rn(g, 2, 7, 5)
        _fd_check(lambda a, b: TF.jeanie(a, b, gamma=0.1, max_shift=1, metric=metric), (q, s),
                  (_rn(g, *q.shape), _rn(g, *s.shape)))
    elif case == "fvm_cost":
        c = torch.rand(2, 3, 2, 6, 7, generator=g, dtype=torch.float64).to(DEV)
        _fd_check(lambda x: TF.fvm_from_cost(x, gamma=0.1), (c,), (_rn(g, *c.shape),))
    elif case == "fvm_features":
        q, s = _rn(g, 2, 4, 6, 5), _rn(g, 2, 7, 5)
        _fd_check(lambda a, b: TF.fvm(a, b, gamma=0.1), (q, s), (_rn(g, *q.shape), _rn(g, *s.shape)))
    else:
        q, s = _rn(g, 2, 4, 6, 5), _rn(g, 2, 3, 7, 5)
        _fd_check(lambda a, b: TF.fvm(a, b, gamma=0.1, metric="sqeuclidean"), (q, s),
                  (_rn(g, *q.shape), _rn(g, *s.shape)))


def _jeanie_with_accumulator(tw, x):
    d, R = tw.functional.jeanie_from_cost(x, gamma=0.1, max_shift=1, return_accumulator=True)
    return d + R.sum((1, 2, 3, 4))


def test_jeanie_accumulator_jvp(tw):
    """Forward mode through the JEANIE accumulator (return_accumulator=True)
    against a central difference."""
    c = torch.rand(1, 2, 2, 4, 5, dtype=torch.float64).to(DEV)
    t = torch.randn(1, 2, 2, 4, 5, dtype=torch.float64).to(DEV)
    _fd_check(lambda x: _jeanie_with_accumulator(tw, x), (c,), (t,))


def test_features_double_backward_normalized(tw):
    """normalize=True evaluates d(X, X): the double backward must give each
    argument slot its own partial derivative.  Checked against a central
    difference of the (native, first-order) gradient along (VX, VY)."""
    g = torch.Generator().manual_seed(21)
    X, Y = _rn(g, 2, 12, 3), _rn(g, 2, 14, 3)
    VX, VY = _rn(g, 2, 12, 3), _rn(g, 2, 14, 3)
    f = lambda a, b: tw.functional.soft_dtw(a, b, gamma=0.3, normalize=True)  # noqa: E731

    def grads(a, b):
        a, b = a.detach().requires_grad_(True), b.detach().requires_grad_(True)
        return torch.autograd.grad(f(a, b).sum(), (a, b))

    x, y = X.clone().requires_grad_(True), Y.clone().requires_grad_(True)
    dX, dY = torch.autograd.grad(f(x, y).sum(), (x, y), create_graph=True)
    hX, hY = torch.autograd.grad((dX * VX).sum() + (dY * VY).sum(), (x, y))
    eps = 1e-6
    gp, gm = grads(X + eps * VX, Y + eps * VY), grads(X - eps * VX, Y - eps * VY)
    _close(hX, ((gp[0] - gm[0]) / (2 * eps)).cpu().numpy(), 1e-6, 1e-5)
    _close(hY, ((gp[1] - gm[1]) / (2 * eps)).cpu().numpy(), 1e-6, 1e-5)


@pytest.mark.parametrize("allow_tf32", [False, True])
def test_features_create_graph_first_order_matches_plain_fp32(tw, allow_tf32):
    """Under create_graph the features backward rebuilds the cost with a cuBLAS
    bmm; it runs in full float32 whatever the caller's TF32 setting, so the
    first-order gradients match the plain native path (tensor-core cost and
    chain rule, 3xTF32) to float32 rounding."""
    g = torch.Generator().manual_seed(21)
    X = torch.randn(3, 96, 64, generator=g).to(DEV)
    Y = torch.randn(3, 80, 64, generator=g).to(DEV)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = allow_tf32
    try:
        x1, y1 = X.clone().requires_grad_(True), Y.clone().requires_grad_(True)
        gx1, gy1 = torch.autograd.grad(tw.functional.soft_dtw(x1, y1, gamma=0.5).sum(), (x1, y1))
        x2, y2 = X.clone().requires_grad_(True), Y.clone().requires_grad_(True)
        gx2, gy2 = torch.autograd.grad(tw.functional.soft_dtw(x2, y2, gamma=0.5).sum(),
                                       (x2, y2), create_graph=True)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    for a, b in ((gx1, gx2), (gy1, gy2)):
        err = (a - b.detach()).abs().max() / a.abs().max()
        assert err < 1e-5, err
