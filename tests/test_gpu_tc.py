"""Tensor-core (tcgen05, 3xTF32) cost and chain-rule kernels against the SIMT
kernels and a float64 PyTorch evaluation of the same formulas
(hibana2077/torchwarp src/torchwarp/csrc/udtw_cuda.cu:379-387, 557-568;
src/torchwarp/udtw/_ops.py:179-183).

Shapes cover D = 64 / 96 / 128 / 256 and ragged D (68), rows and columns that
are not multiples of the 128-cell tiles, and cells with an exactly zero cost
(masked out of the gradient).
"""

import pytest
import torch

from torchwarp_b200 import _native as nat

pytestmark = pytest.mark.gpu

SHAPES = [(3, 200, 300, 64), (2, 129, 260, 96), (2, 64, 128, 128), (1, 300, 132, 68),
          (2, 130, 140, 256), (1, 1, 4, 64), (5, 33, 36, 64)]


def _inputs(B, N, M, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(B, N, D, device="cuda", generator=g)
    Y = torch.randn(B, M, D, device="cuda", generator=g)
    vx = 0.25 + torch.rand(B, N, device="cuda", generator=g)
    vy = 0.25 + torch.rand(B, M, device="cuda", generator=g)
    return X, Y, vx, vy


def _env(monkeypatch, simt):
    if simt:
        monkeypatch.setenv("TW_COST_SIMT", "1")
    else:
        monkeypatch.delenv("TW_COST_SIMT", raising=False)


def _cost(X, Y, vx, vy, beta, eps):
    B, N, D = X.shape
    M = Y.shape[1]
    C = torch.empty(B, N, M, device="cuda")
    Q = torch.empty(B, N, M, device="cuda") if vx is not None else None
    st = nat.lib().tw_udtw_cost_f32(nat.ptr(X), nat.ptr(Y), nat.ptr(vx), nat.ptr(vy), B, N, M, D,
                                    beta, eps, nat.ptr(C), nat.ptr(Q), nat.stream_of(X))
    nat.check(st, "tw_udtw_cost_f32")
    torch.cuda.synchronize()
    return C, Q


def _cost_ref(X, Y, vx, vy, beta, eps):
    X, Y = X.double(), Y.double()
    sq = (X * X).sum(-1)[:, :, None] + (Y * Y).sum(-1)[:, None, :] - 2 * X @ Y.transpose(1, 2)
    sq = sq.clamp_min(0)
    if vx is None:
        return sq, None
    var = (0.5 * (vx.double()[:, :, None] + vy.double()[:, None, :])).clamp_min(eps)
    return sq / var, beta * torch.log(var)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("var", [False, True])
def test_tc_cost(shape, var, monkeypatch):
    X, Y, vx, vy = _inputs(*shape, seed=sum(shape))
    if not var:
        vx = vy = None
    _env(monkeypatch, False)
    C, Q = _cost(X, Y, vx, vy, 1.0, 1e-8)
    assert nat.lib().tw_device_error() == 0
    _env(monkeypatch, True)
    Cs, Qs = _cost(X, Y, vx, vy, 1.0, 1e-8)
    Cr, Qr = _cost_ref(X, Y, vx, vy, 1.0, 1e-8)
    D = shape[3]
    # fp32 evaluation of |x|^2 + |y|^2 - 2 x.y: absolute error ~ 2^-23 * 4D
    atol = 4 * D * 2.0 ** -20
    torch.testing.assert_close(C.double(), Cr, rtol=1e-5, atol=atol)
    torch.testing.assert_close(C, Cs, rtol=1e-5, atol=atol)
    if var:
        # the tensor-core epilogue takes beta ln(var) from the hardware log2
        # (relative error ~2^-22); the SIMT kernel calls logf
        torch.testing.assert_close(Q.double(), Qr, rtol=2e-6, atol=2e-6)
        torch.testing.assert_close(Q, Qs, rtol=2e-6, atol=2e-6)


def test_tc_cost_self_distance_is_zero_on_the_diagonal(monkeypatch):
    # d(X, X): the diagonal sq_raw cancels to ~0 and must clamp to exactly 0
    _env(monkeypatch, False)
    X, _, _, _ = _inputs(2, 256, 256, 64, seed=5)
    C, _ = _cost(X, X, None, None, 0.0, 1e-8)
    diag = torch.diagonal(C, dim1=1, dim2=2)
    assert float(diag.abs().max()) < 1e-3
    assert nat.lib().tw_device_error() == 0


def _grad(X, Y, vx, vy, C, dC, dQ, beta, eps):
    B, N, D = X.shape
    M = Y.shape[1]
    dX = torch.full_like(X, float("nan"))
    dY = torch.full_like(Y, float("nan"))
    dvx = torch.full_like(vx, float("nan")) if vx is not None else None
    dvy = torch.full_like(vy, float("nan")) if vy is not None else None
    st = nat.lib().tw_udtw_features_grad_f32(
        nat.ptr(X), nat.ptr(Y), nat.ptr(vx), nat.ptr(vy), nat.ptr(C), nat.ptr(dC), nat.ptr(dQ),
        B, N, M, D, beta, eps, nat.ptr(dX), nat.ptr(dY), nat.ptr(dvx), nat.ptr(dvy),
        nat.stream_of(X))
    nat.check(st, "tw_udtw_features_grad_f32")
    torch.cuda.synchronize()
    return dX, dY, dvx, dvy


def _grad_ref(X, Y, vx, vy, C, dC, dQ, beta, eps):
    X, Y, C, dC = X.double(), Y.double(), C.double(), dC.double()
    if vx is None:
        var = torch.ones_like(C)
        var_raw = var
    else:
        var_raw = 0.5 * (vx.double()[:, :, None] + vy.double()[:, None, :])
        var = var_raw.clamp_min(eps)
    S = torch.where(C > 0, dC / var, torch.zeros_like(C))
    dX = -2 * S @ Y + 2 * X * S.sum(2, keepdim=True)
    dY = -2 * S.transpose(1, 2) @ X + 2 * Y * S.sum(1)[:, :, None]
    if vx is None:
        return dX, dY, None, None
    q = dQ.double() if dQ is not None else torch.zeros_like(C)
    dvar = torch.where(var_raw > eps, (beta * q - dC * C) / var, torch.zeros_like(C))
    return dX, dY, 0.5 * dvar.sum(2), 0.5 * dvar.sum(1)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("mode", ["sdtw", "udtw", "udtw_no_dq"])
def test_tc_grad(shape, mode, monkeypatch):
    B, N, M, D = shape
    X, Y, vx, vy = _inputs(*shape, seed=7 * sum(shape))
    g = torch.Generator(device="cuda").manual_seed(11)
    C = torch.rand(B, N, M, device="cuda", generator=g) * 100
    C[C < 5] = 0.0  # exact zeros are masked out of dsq
    dC = torch.randn(B, N, M, device="cuda", generator=g)
    dQ = torch.randn(B, N, M, device="cuda", generator=g)
    if mode == "sdtw":
        vx = vy = dQ = None
    elif mode == "udtw_no_dq":
        dQ = None
    beta, eps = 0.7, 1e-8
    _env(monkeypatch, False)
    got = _grad(X, Y, vx, vy, C, dC, dQ, beta, eps)
    assert nat.lib().tw_device_error() == 0
    _env(monkeypatch, True)
    simt = _grad(X, Y, vx, vy, C, dC, dQ, beta, eps)
    ref = _grad_ref(X, Y, vx, vy, C, dC, dQ, beta, eps)
    for a, s, r in zip(got, simt, ref):
        if r is None:
            assert a is None
            continue
        assert torch.isfinite(a).all()
        scale = float(r.abs().max()) + 1.0
        torch.testing.assert_close(a.double(), r, rtol=1e-4, atol=2e-5 * scale)
        torch.testing.assert_close(a, s, rtol=1e-4, atol=2e-5 * scale)


def test_tc_grad_is_deterministic(monkeypatch):
    _env(monkeypatch, False)
    B, N, M, D = 4, 256, 384, 64
    X, Y, vx, vy = _inputs(B, N, M, D, seed=3)
    C = torch.rand(B, N, M, device="cuda") + 0.1
    dC = torch.randn(B, N, M, device="cuda")
    a = _grad(X, Y, None, None, C, dC, None, 0.0, 1e-8)
    b = _grad(X, Y, None, None, C, dC, None, 0.0, 1e-8)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_soft_dtw_features_path_uses_tensor_cores(monkeypatch, orc):
    """soft_dtw at D = 64 (tensor-core cost and chain rule) against the
    float64 oracle: value and gradient errors no larger than those of the
    fp32 SIMT path on the same inputs (both are fp32 dynamic programs; only
    the contraction differs)."""
    import numpy as np

    import torchwarp_b200 as tw
    g = torch.Generator().manual_seed(2)
    X = torch.randn(4, 160, 64, generator=g)
    Y = torch.randn(4, 192, 64, generator=g)
    od, odx, ody = orc.soft_dtw(X.double().numpy(), Y.double().numpy(), gamma=1.0)
    errs = []
    for simt in (False, True):
        _env(monkeypatch, simt)
        x = X.cuda().requires_grad_(True)
        y = Y.cuda().requires_grad_(True)
        d = tw.functional.soft_dtw(x, y, gamma=1.0)
        d.sum().backward()
        ed = np.abs(d.detach().double().cpu().numpy() - od).max() / np.abs(od).max()
        ex = np.abs(x.grad.double().cpu().numpy() - odx).max() / np.abs(odx).max()
        ey = np.abs(y.grad.double().cpu().numpy() - ody).max() / np.abs(ody).max()
        errs.append((ed, ex, ey))
    assert nat.lib().tw_device_error() == 0
    (tc_d, tc_x, tc_y), (si_d, si_x, si_y) = errs
    assert tc_d < 1e-5 and tc_x < 1e-4 and tc_y < 1e-4, errs
    assert tc_d <= 2 * si_d + 1e-7 and tc_x <= 2 * si_x + 1e-6 and tc_y <= 2 * si_y + 1e-6, errs


# ------------------------------------------- squared-Euclidean cost + mask

def _sq_cost(X, Y):
    B, N, D = X.shape
    M = Y.shape[1]
    C = torch.empty(B, N, M, device="cuda", dtype=X.dtype)
    mask = torch.empty(B, (M + 31) // 32, (N + 3) // 4 * 4, device="cuda", dtype=torch.int32)
    fn = getattr(nat.lib(), "tw_sqeuclid_cost_" + nat.suffix(X.dtype))
    nat.check(fn(nat.ptr(X), nat.ptr(Y), B, N, M, D, nat.ptr(C), nat.ptr(mask),
                 nat.stream_of(X)), "tw_sqeuclid_cost")
    torch.cuda.synchronize()
    return C, mask


def _pack_positive(C):
    """[B, N, M] cost -> [B, ceil(M/32), 4 ceil(N/4)] words with bit j&31 set
    where C > 0 (padding rows zero)."""
    B, N, M = C.shape
    MW = (M + 31) // 32
    NP = (N + 3) // 4 * 4
    pos = torch.zeros(B, NP, MW * 32, dtype=torch.int64, device=C.device)
    pos[:, :N, :M] = (C > 0).long()
    w = (pos.view(B, NP, MW, 32) << torch.arange(32, device=C.device)).sum(-1)
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)
    return w.transpose(1, 2).contiguous()


@pytest.mark.parametrize("shape", SHAPES + [(2, 70, 45, 8), (3, 33, 100, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("simt", [False, True])
def test_sq_cost_and_mask(shape, dtype, simt, monkeypatch):
    if dtype == torch.float64 and simt:
        pytest.skip("float64 always runs the SIMT kernels")
    _env(monkeypatch, simt)
    X, Y, _, _ = _inputs(*shape, seed=3 * sum(shape))
    X, Y = X.to(dtype), Y.to(dtype)
    # exact duplicates: sq_raw <= 0 there, so the mask has zeros to find
    n = min(X.shape[1], Y.shape[1])
    Y[:, : n // 2] = X[:, : n // 2]
    C, mask = _sq_cost(X, Y)
    assert nat.lib().tw_device_error() == 0
    Cu, _ = _cost(X.float(), Y.float(), None, None, 0.0, 1e-8) if dtype == torch.float32 else (
        None, None)
    if Cu is not None:
        assert torch.equal(C, Cu)
    assert torch.equal(mask, _pack_positive(C))


def _unpack_mask(mask, N, M):
    w = mask.to(torch.int64) & 0xFFFFFFFF
    j = torch.arange(M, device=mask.device)
    bits = (w[:, j // 32, :N] >> (j % 32)[None, :, None]) & 1
    return bits.transpose(1, 2).bool().contiguous()


@pytest.mark.parametrize("shape", SHAPES + [(2, 70, 45, 8)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("smem_s", [False, True])
def test_sq_grad_premasked(shape, dtype, smem_s, monkeypatch):
    """With a null mask the chain rule takes d_cost as already masked; on
    S = d_cost * mask it reproduces the mask path (float64 exactly, float32
    within its accumulation rounding)."""
    if dtype == torch.float64 and smem_s:
        pytest.skip("float64 always runs the SIMT kernels")
    _env(monkeypatch, False)
    if smem_s:
        monkeypatch.setenv("TW_GRAD_SMEM_S", "1")
    B, N, M, D = shape
    X, Y, _, _ = _inputs(*shape, seed=7 * sum(shape))
    X, Y = X.to(dtype), Y.to(dtype)
    n = min(N, M)
    Y[:, : n // 3] = X[:, : n // 3]
    C, mask = _sq_cost(X, Y)
    dC = torch.randn(B, N, M, device="cuda", dtype=dtype)
    S = torch.where(_unpack_mask(mask, N, M), dC, torch.zeros_like(dC)).contiguous()
    fn = getattr(nat.lib(), "tw_sqeuclid_grad_" + nat.suffix(dtype))
    outs = []
    for m, d in ((mask, dC), (None, S)):
        dX = torch.empty_like(X)
        dY = torch.empty_like(Y)
        nat.check(fn(nat.ptr(X), nat.ptr(Y), None if m is None else nat.ptr(m), nat.ptr(d), B, N,
                     M, D, nat.ptr(dX), nat.ptr(dY), nat.stream_of(X)), "tw_sqeuclid_grad")
        outs.append((dX, dY))
    torch.cuda.synchronize()
    assert nat.lib().tw_device_error() == 0
    (aX, aY), (bX, bY) = outs
    if dtype == torch.float64:
        assert torch.equal(aX, bX) and torch.equal(aY, bY)
    else:
        for a, b in ((aX, bX), (aY, bY)):
            err = ((a - b).abs() / (a.abs() + 1.0)).max().item()
            assert err < 2e-6, err


@pytest.mark.parametrize("shape", SHAPES + [(2, 70, 45, 8)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_sq_grad_mask_equals_cost_path(shape, dtype, monkeypatch):
    """The chain rule from the mask is bit-identical to the one from the cost."""
    _env(monkeypatch, False)
    B, N, M, D = shape
    X, Y, _, _ = _inputs(*shape, seed=5 * sum(shape))
    X, Y = X.to(dtype), Y.to(dtype)
    n = min(N, M)
    Y[:, : n // 3] = X[:, : n // 3]
    C, mask = _sq_cost(X, Y)
    dC = torch.randn(B, N, M, device="cuda", dtype=dtype)
    dX = torch.empty_like(X)
    dY = torch.empty_like(Y)
    fn = getattr(nat.lib(), "tw_sqeuclid_grad_" + nat.suffix(dtype))
    nat.check(fn(nat.ptr(X), nat.ptr(Y), nat.ptr(mask), nat.ptr(dC), B, N, M, D, nat.ptr(dX),
                 nat.ptr(dY), nat.stream_of(X)), "tw_sqeuclid_grad")
    fn2 = getattr(nat.lib(), "tw_udtw_features_grad_" + nat.suffix(dtype))
    rX = torch.empty_like(X)
    rY = torch.empty_like(Y)
    nat.check(fn2(nat.ptr(X), nat.ptr(Y), None, None, nat.ptr(C), nat.ptr(dC), None, B, N, M, D,
                  0.0, 1e-8, nat.ptr(rX), nat.ptr(rY), None, None, nat.stream_of(X)),
              "tw_udtw_features_grad")
    torch.cuda.synchronize()
    assert nat.lib().tw_device_error() == 0
    assert torch.equal(dX, rX) and torch.equal(dY, rY)
