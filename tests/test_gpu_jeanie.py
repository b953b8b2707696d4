"""JEANIE / FVM / cost builders / argmin paths on B200 vs golden vectors and the oracle.

float64 tolerances are the reference tests' (atol 1e-10, rtol 1e-9:
tests/test_jeanie.py:23,33-34 of hibana2077/torchwarp); argmin paths must be
identical cell for cell.
"""

import numpy as np
import pytest
import torch

import golden_data as G

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-10, 1e-9
DEV = "cuda"


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


def _vg(fn, x):
    c = _t(x).requires_grad_(True)
    out = fn(c)
    out.sum().backward()
    return out, c.grad


@pytest.mark.parametrize("K,T,U", G.JEANIE_1D_SHAPES)
@pytest.mark.parametrize("shift", G.JEANIE_1D_SHIFTS)
def test_jeanie_1d_golden(tw, K, T, U, shift):
    ref = G.official("jeanie.jeanie_1d", K=K, T=T, U=U, shift=shift)
    v, g = _vg(lambda c: tw.functional.jeanie_from_cost(c[None], gamma=0.1, max_shift=shift)[0],
               ref["cost"])
    _close(v, ref["value"])
    _close(g, ref["grad"])
    _, acc = tw.functional.jeanie_from_cost(_t(ref["cost"][None]), gamma=0.1, max_shift=shift,
                                            return_accumulator=True)
    _close(acc[0], ref["accumulator"])


@pytest.mark.parametrize("K1,K2,T,U", G.JEANIE_2D_SHAPES)
@pytest.mark.parametrize("s_az,s_alt", G.JEANIE_2D_SHIFTS)
def test_jeanie_2d_golden(tw, K1, K2, T, U, s_az, s_alt):
    ref = G.official("jeanie.jeanie_2d", K1=K1, K2=K2, T=T, U=U, s_az=s_az, s_alt=s_alt)
    v, g = _vg(lambda c: tw.functional.jeanie_from_cost(c[None], gamma=0.1,
                                                        max_shift=(s_az, s_alt))[0], ref["cost"])
    _close(v, ref["value"])
    _close(g, ref["grad"])


def test_jeanie_batched_golden(tw):
    ref = G.official("jeanie.batched")
    _close(tw.functional.jeanie_from_cost(_t(ref["cost_1d"]), gamma=0.1, max_shift=1),
           ref["value_1d"])
    _close(tw.functional.jeanie_from_cost(_t(ref["cost_2d"]), gamma=0.1, max_shift=(1, 1)),
           ref["value_2d"])


@pytest.mark.parametrize("name,shape", G.FVM_CASES)
def test_fvm_golden(tw, name, shape):
    ref = G.official("jeanie.fvm", name=name)
    v, g = _vg(lambda c: tw.functional.fvm_from_cost(c[None], gamma=0.1)[0], ref["cost"])
    _close(v, ref["value"])
    _close(g, ref["grad"])
    _close(tw.functional.fvm_from_cost(_t(ref["batch"]), gamma=0.1), ref["batch_value"])


@pytest.mark.parametrize("name,shape,shift", G.LARGE_COST)
def test_large_golden(tw, name, shape, shift):
    ref = G.official("jeanie.large", name=name, shape=shape)
    TF = tw.functional
    if name == "soft_dtw":
        fn = lambda c: TF.soft_dtw_from_cost(c[None], gamma=0.1)[0]  # noqa: E731
    elif name.startswith("fvm"):
        fn = lambda c: TF.fvm_from_cost(c[None], gamma=0.1)[0]  # noqa: E731
    else:
        fn = lambda c: TF.jeanie_from_cost(c[None], gamma=0.1, max_shift=shift)[0]  # noqa: E731
    v, g = _vg(fn, ref["cost"])
    _close(v, ref["value"])
    _close(g, ref["grad"])


@pytest.mark.parametrize("name", ["euclidean_cost", "squared_euclidean_cost", "rbf_cost"])
def test_distances_golden(tw, name):
    ref = G.official("jeanie.distance", name=name)
    q, s = _t(ref["q"]).requires_grad_(), _t(ref["s"]).requires_grad_()
    out = getattr(tw, name)(q, s)
    g = torch.autograd.grad(out.sum(), (q, s))
    _close(out, ref["value"])
    for a, b in zip(g, ref["grads"]):
        _close(a, b)
    _close(getattr(tw, name)(_t(ref["qb"]), _t(ref["sb"])), ref["batch_value"])


def _rbf_definition(q, s, sigma):
    diff = q.unsqueeze(-2) - s.unsqueeze(-3)
    return (2.0 - 2.0 * torch.exp(-sigma * diff.pow(2))).sum(-1)


@pytest.mark.parametrize("qshape,sshape,sigma", [
    ((2, 5, 3), (2, 7, 3), 0.5),             # two sequences
    ((3, 4, 6, 8), (3, 37, 8), 0.3),         # JEANIE layout, U across support chunks
    ((2, 3, 1, 5, 7), (2, 1, 4, 9, 7), 1.2),  # FVM with support-side viewpoints (broadcast)
    ((2, 15, 10, 256), (2, 10, 256), 0.5),   # cfg3 feature size
])
def test_rbf_cost_native_vs_definition(tw, qshape, sshape, sigma):
    """The native rbf cost and its gradient against the reference's PyTorch
    definition (jeanie/distances.py:41-51), float64."""
    g = torch.Generator().manual_seed(sum(qshape) + sum(sshape))
    q = torch.randn(*qshape, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    s = torch.randn(*sshape, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    if len(sshape) == len(qshape):
        want = _rbf_definition(q, s, sigma)
    else:
        want = _rbf_definition(q, s.unsqueeze(-3), sigma)
    got = tw.rbf_cost(q, s, sigma=sigma)
    assert got.shape == want.shape
    w = torch.randn(want.shape, generator=g, dtype=torch.float64).to(DEV)
    gq, gs = torch.autograd.grad((got * w).sum(), (q, s))
    wq, ws = torch.autograd.grad((want * w).sum(), (q, s))
    _close(got, want.detach().cpu().numpy())
    _close(gq, wq.cpu().numpy())
    _close(gs, ws.cpu().numpy())


def test_rbf_cost_fp32_and_deterministic(tw):
    g = torch.Generator().manual_seed(9)
    q = torch.randn(8, 150, 64, generator=g).to(DEV).requires_grad_(True)
    s = torch.randn(8, 10, 64, generator=g).to(DEV).requires_grad_(True)
    got = tw.rbf_cost(q, s)
    want = _rbf_definition(q.double(), s.double(), 0.5)
    err = (got.double() - want).abs().max() / want.abs().max()
    assert err < 1e-6, err
    w = torch.randn(got.shape, generator=g).to(DEV)
    g1 = torch.autograd.grad((got * w).sum(), (q, s), retain_graph=True)
    g2 = torch.autograd.grad((got * w).sum(), (q, s))
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))


def test_end_to_end_golden(tw):
    ref = G.official("jeanie.end_to_end")
    q, s = _t(ref["q"]).requires_grad_(), _t(ref["s"]).requires_grad_()
    d = tw.functional.jeanie_from_cost(tw.euclidean_cost(q[None], s[None]), gamma=0.1,
                                       max_shift=1)[0]
    g = torch.autograd.grad(d, (q, s))
    _close(d, ref["value"])
    for a, b in zip(g, ref["grads"]):
        _close(a, b)


@pytest.mark.parametrize("metric", G.METRICS)
@pytest.mark.parametrize("K,T,U,shift", G.FEATURES_1D)
def test_jeanie_features_1d_golden(tw, metric, K, T, U, shift):
    ref = G.official("jeanie.features_1d", metric=metric, K=K, T=T, U=U, shift=shift)
    qb, sb = _t(ref["q"]).requires_grad_(), _t(ref["s"]).requires_grad_()
    d = tw.functional.jeanie(qb, sb, gamma=0.1, max_shift=shift, metric=metric)
    g = torch.autograd.grad(d.sum(), (qb, sb))
    _close(d, ref["value"])
    for a, b in zip(g, ref["grads"]):
        _close(a, b)


@pytest.mark.parametrize("metric", ["euclidean", "sqeuclidean"])
def test_jeanie_features_2d_golden(tw, metric):
    ref = G.official("jeanie.features_2d", metric=metric)
    qb, sb = _t(ref["q"]).requires_grad_(), _t(ref["s"]).requires_grad_()
    d, acc = tw.functional.jeanie(qb, sb, gamma=0.1, max_shift=(1, 1), metric=metric,
                                  return_accumulator=True)
    g = torch.autograd.grad(d.sum(), (qb, sb))
    _close(d, ref["value"])
    for a, b in zip(g, ref["grads"]):
        _close(a, b)
    _close(acc[0], ref["accumulator"])


@pytest.mark.parametrize("K,T,U,shift", G.ACCUMULATOR_COST)
def test_accumulator_cost_golden(tw, K, T, U, shift):
    ref = G.official("parity.accumulator_cost", K=K, T=T, U=U, shift=shift)
    c = _t(ref["cost"]).requires_grad_()
    d, R = tw.functional.jeanie_from_cost(c[None], gamma=0.3, max_shift=shift,
                                          return_accumulator=True)
    (g,) = torch.autograd.grad(d[0] + 0.1 * (R ** 2).mean(), c)
    _close(g, ref["grad"])


def test_accumulator_2d_golden(tw):
    ref = G.official("parity.accumulator_2d")
    c = _t(ref["cost"]).requires_grad_()
    d, R = tw.functional.jeanie_from_cost(c[None], gamma=0.3, max_shift=(1, 1),
                                          return_accumulator=True)
    (g,) = torch.autograd.grad(d[0] + R.sin().sum(), c)
    _close(g, ref["grad"])


SCALED = ["jeanie_cfg3", "jeanie_2d", "jeanie_cost_big", "fvm_cfg4", "fvm_cost_cfg4"]


@pytest.mark.parametrize("name", SCALED)
def test_scaled_reference_backend(tw, name):
    ins, kw, vals, grads = G.scaled(name)
    xs = [_t(x).requires_grad_(True) for x in ins]
    TF = tw.functional
    if name.startswith("jeanie_cost"):
        d = TF.jeanie_from_cost(xs[0], **kw)
    elif name.startswith("jeanie"):
        d = TF.jeanie(xs[0], xs[1], **kw)
    elif name.startswith("fvm_cost"):
        d = TF.fvm_from_cost(xs[0], **kw)
    else:
        d = TF.fvm(xs[0], xs[1], **kw)
    d.sum().backward()
    _close(d, vals[0])
    for x, g in zip(xs, grads):
        _close(x.grad, g, atol=1e-9, rtol=1e-8)


# Shapes across the diagonal-length and viewpoint ranges (reference
# tests/test_jeanie.py:188-214 sweeps K up to 64 and T, U up to 300).
KERNEL_SHAPES = [(1, 257, 300, 0), (5, 205, 220, 2), (5, 300, 200, 1), (16, 130, 140, 2),
                 (64, 128, 130, 1)]


@pytest.mark.parametrize("K,T,U,shift", KERNEL_SHAPES)
def test_kernel_shapes_vs_oracle(tw, orc, K, T, U, shift):
    g = torch.Generator().manual_seed(K * T * U)
    cost = torch.rand(1, K, T, U, generator=g, dtype=torch.float64)
    v, gr = _vg(lambda c: tw.functional.jeanie_from_cost(c, gamma=0.1, max_shift=shift),
                cost.numpy())
    od, _, odc = orc.jeanie_from_cost(cost.numpy(), gamma=0.1, max_shift=shift)
    _close(v, od)
    _close(gr, odc, atol=1e-9, rtol=1e-8)


@pytest.mark.parametrize("metric", ["euclidean", "sqeuclidean"])
def test_features_vs_oracle(tw, orc, metric):
    g = torch.Generator().manual_seed(3)
    q = torch.randn(3, 6, 40, 70, generator=g, dtype=torch.float64)
    s = torch.randn(3, 45, 70, generator=g, dtype=torch.float64)
    qq, ss = _t(q).requires_grad_(), _t(s).requires_grad_()
    d = tw.functional.jeanie(qq, ss, gamma=0.1, max_shift=2, metric=metric)
    d.sum().backward()
    od, _, odq, ods = orc.jeanie(q.numpy(), s.numpy(), gamma=0.1, max_shift=2, metric=metric)
    _close(d, od)
    _close(qq.grad, odq, atol=1e-9, rtol=1e-8)
    _close(ss.grad, ods, atol=1e-9, rtol=1e-8)


@pytest.mark.parametrize("metric", G.METRICS)
@pytest.mark.parametrize("qshape,sshape", [((2, 4, 6, 5), (2, 3, 7, 5)),
                                           ((2, 2, 3, 6, 5), (2, 3, 2, 7, 5))])
def test_fvm_support_viewpoints(tw, orc, metric, qshape, sshape):
    """Support-side viewpoints: the cost of every (query, support) viewpoint
    pair comes from one query/support launch over all K' U support frames."""
    g = torch.Generator().manual_seed(7)
    q = torch.randn(*qshape, generator=g, dtype=torch.float64)
    s = torch.randn(*sshape, generator=g, dtype=torch.float64)
    qq, ss = _t(q).requires_grad_(), _t(s).requires_grad_()
    d = tw.functional.fvm(qq, ss, gamma=0.1, metric=metric)
    d.sum().backward()
    od, odq, ods = orc.fvm(q.numpy(), s.numpy(), gamma=0.1, metric=metric)
    _close(d, od)
    _close(qq.grad, odq)
    _close(ss.grad, ods)


def test_features_zero_distance_grad_is_finite(tw):
    q = torch.ones(1, 2, 3, 4, dtype=torch.float64, device=DEV, requires_grad=True)
    s = torch.ones(1, 3, 4, dtype=torch.float64, device=DEV, requires_grad=True)
    tw.functional.jeanie(q, s, gamma=0.1, max_shift=1).sum().backward()
    assert torch.isfinite(q.grad).all() and torch.isfinite(s.grad).all()


def test_float32_accuracy(tw, orc):
    g = torch.Generator().manual_seed(0)
    cost = torch.rand(8, 5, 12, 15, generator=g, dtype=torch.float64)
    c32 = cost.float().to(DEV).requires_grad_()
    v = tw.functional.jeanie_from_cost(c32, gamma=0.1, max_shift=1)
    v.sum().backward()
    od, _, odc = orc.jeanie_from_cost(cost.numpy(), gamma=0.1, max_shift=1)
    for a, b in ((v, od), (c32.grad, odc)):
        err = np.abs(a.detach().double().cpu().numpy() - b).max() / np.abs(b).max()
        assert err < 1e-4, err


def test_jeanie_deterministic(tw):
    g = torch.Generator().manual_seed(0)
    q = torch.randn(4, 16, 40, 8, generator=g).to(DEV)
    s = torch.randn(4, 45, 8, generator=g).to(DEV)

    def run():
        a, b = q.clone().requires_grad_(), s.clone().requires_grad_()
        d = tw.functional.jeanie(a, b, gamma=0.1, max_shift=1)
        d.sum().backward()
        return d.detach(), a.grad, b.grad

    first = run()
    for _ in range(2):
        assert all(torch.equal(x, y) for x, y in zip(run(), first))


# ----------------------------------------------------------------- paths

@pytest.mark.parametrize("K,T,U,shift,start", [(1, 9, 12, 0, None), (3, 4, 5, 1, None),
                                                 (3, 4, 5, 2, 1), (5, 30, 41, 1, None),
                                                 (7, 20, 20, 7, 3)])
def test_optimal_path_bit_exact(tw, orc, K, T, U, shift, start):
    g = torch.Generator().manual_seed(K + T + U)
    cost = torch.rand(3, K, T, U, generator=g, dtype=torch.float64)
    got = tw.paths.optimal_path(cost.to(DEV), max_shift=shift, start_view=start)
    for b in range(3):
        assert got[b] == orc.optimal_path(cost[b].numpy(), shift, start)


def test_optimal_path_ties_follow_reference_order(tw, orc):
    cost = torch.zeros(2, 3, 6, 7, dtype=torch.float64)  # every path ties
    cost[1, :, 2:4, :] = 1.0
    got = tw.paths.optimal_path(cost.to(DEV), max_shift=1)
    for b in range(2):
        assert got[b] == orc.optimal_path(cost[b].numpy(), 1, None)


def test_path_matrix_is_gradient(tw):
    g = torch.Generator().manual_seed(0)
    cost = torch.rand(3, 9, 12, generator=g, dtype=torch.float64).to(DEV)
    a = tw.paths.soft_dtw(cost, gamma=1e-3)
    for b in range(3):
        p = a.optimal_path[b]
        assert p[0] == (0, 0) and p[-1] == (8, 11)
        assert float(a.path_matrix[b, 0, 0]) == pytest.approx(1.0, abs=1e-6)


# ------------------------- fp32 warp-per-row query/support cost and gradient

def _qs_ref(q, s, metric):
    q, s = q.double(), s.double()
    raw = (q * q).sum(-1)[:, :, None] + (s * s).sum(-1)[:, None, :] - 2 * q @ s.transpose(1, 2)
    sq = raw.clamp_min(0)
    return torch.where(raw > 0, sq.sqrt(), torch.zeros_like(sq)) if metric == 1 else sq


@pytest.mark.parametrize("R,U,D", [(150, 10, 256), (490, 10, 256), (37, 3, 64), (64, 16, 128),
                                   (20, 12, 100), (9, 7, 252), (33, 10, 36)])
@pytest.mark.parametrize("metric", [0, 1])
def test_qs_fast_fp32(R, U, D, metric):
    """The fp32 query/support cost and its chain rule (warp-per-row kernels for
    U <= 16, D <= 256) against a float64 torch evaluation of the same formulas
    (jeanie/distances.py:15-38; zero gradient where the cost is 0)."""
    from torchwarp_b200 import _native as nat
    B = 6
    g = torch.Generator(device=DEV).manual_seed(R + U + D)
    q = torch.randn(B, R, D, device=DEV, generator=g)
    s = torch.randn(B, U, D, device=DEV, generator=g)
    q[:, 0] = s[:, 0]  # an exactly zero cost
    cost = torch.empty(B, R, U, device=DEV)
    st = nat.stream_of(q)
    nat.check(nat.lib().tw_qs_cost_f32(nat.ptr(q), nat.ptr(s), B, R, U, D, metric,
                                       nat.ptr(cost), st), "qs cost")
    torch.cuda.synchronize()
    ref = _qs_ref(q, s, metric)
    # fp32 rounding of |q|^2 + |s|^2 - 2 q.s is ~1e-4 here; its square root (metric 1)
    # near a zero distance is ~1e-2
    torch.testing.assert_close(cost.double(), ref, rtol=1e-5, atol=2e-2 if metric else 1e-3 * D / 8)
    dcost = torch.randn(B, R, U, device=DEV, generator=g)
    dq, ds = torch.empty_like(q), torch.empty_like(s)
    nat.check(nat.lib().tw_qs_cost_grad_f32(nat.ptr(q), nat.ptr(s), nat.ptr(cost), nat.ptr(dcost),
                                            B, R, U, D, metric, nat.ptr(dq), nat.ptr(ds), st),
              "qs grad")
    torch.cuda.synchronize()
    c64 = cost.double()
    dc = dcost.double()
    dsq = torch.where(c64 > 0, dc * 0.5 / c64 if metric == 1 else dc, torch.zeros_like(dc))
    q64, s64 = q.double(), s.double()
    rdq = 2 * q64 * dsq.sum(2, keepdim=True) - 2 * dsq @ s64
    rds = 2 * s64 * dsq.sum(1)[:, :, None] - 2 * dsq.transpose(1, 2) @ q64
    for got, want in ((dq, rdq), (ds, rds)):
        scale = float(want.abs().max()) + 1.0
        torch.testing.assert_close(got.double(), want, rtol=1e-4, atol=1e-5 * scale)
