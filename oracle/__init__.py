"""CPU oracle: float64 restatement of torchwarp's alignment algorithms.

TEST INFRASTRUCTURE ONLY.  The dynamic programs run in ``oracle.c`` (plain C,
float64, loaded with ctypes); this module composes them with numpy into the
same public semantics as the reference's functional API
(hibana2077/torchwarp ``src/torchwarp/functional.py``), forward values and
first-order gradients.  Only tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import it; the product never does.

Conventions: every function takes and returns float64 numpy arrays.  A
``*_grad`` function returns the gradients of ``sum(g_out * out)`` (plus
``sum(g_pen * pen)`` for uDTW) with respect to the listed inputs.
"""

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

_dp = ctypes.POINTER(ctypes.c_double)
_ip = ctypes.POINTER(ctypes.c_int)


def build():
    """Compile oracle.c into oracle/_build/liboracle.so (gcc, no GPU)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        i, d = ctypes.c_int, ctypes.c_double
        L.orc_udtw_forward.argtypes = [_dp, _dp, i, i, i, d, d, _dp, _dp, _dp, _dp]
        L.orc_udtw_backward.argtypes = [_dp, _dp, _dp, _dp, _dp, _dp, i, i, i, d, _dp, _dp]
        L.orc_jeanie_forward.argtypes = [_dp, i, i, i, i, i, i, i, d, _dp, _dp]
        L.orc_jeanie_backward.argtypes = [_dp, _dp, _dp, _dp, i, i, i, i, i, i, i, d, _dp]
        L.orc_optimal_path.argtypes = [_dp, i, i, i, i, i, _ip]
        L.orc_optimal_path.restype = i
        _lib = L
    return _lib


def _c(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _p(a):
    return None if a is None else a.ctypes.data_as(_dp)


# ----------------------------------------------------------- dynamic programs

def udtw_dp(C, Q, gamma, band=0.0):
    """uDTW DP on cost/penalty [B,N,M] (udtw/_torch_dp.py:14-42).
    Returns (out_r [B], out_p [B], R, P)."""
    C, Q = _c(C), (None if Q is None else _c(Q))
    B, N, M = C.shape
    out_r, out_p = np.empty(B), np.empty(B)
    R, P = np.empty_like(C), np.empty_like(C)
    lib().orc_udtw_forward(_p(C), _p(Q), B, N, M, float(gamma), float(band),
                           _p(out_r), _p(out_p), _p(R), _p(P))
    return out_r, out_p, R, P


def udtw_dp_grad(C, Q, gamma, band, g_r, g_p=None):
    """(dC, dQ) of sum(g_r * out_r + g_p * out_p) (udtw/_torch_dp.py:45-76)."""
    C = _c(C)
    Qc = None if Q is None else _c(Q)
    B, N, M = C.shape
    _, _, R, P = udtw_dp(C, Qc, gamma, band)
    g_r = _c(np.broadcast_to(g_r, (B,)))
    g_p = None if g_p is None else _c(np.broadcast_to(g_p, (B,)))
    dC, dQ = np.empty_like(C), np.empty_like(C)
    lib().orc_udtw_backward(_p(C), _p(Qc), _p(R), _p(P), _p(g_r), _p(g_p), B, N, M,
                            float(gamma), _p(dC), _p(dQ))
    return dC, dQ


def jeanie_dp(C5, s1, s2, gamma):
    """JEANIE DP on [B,K1,K2,T,U] (jeanie/_torch_dp.py:14-38) -> (out [B], R)."""
    C5 = _c(C5)
    B, K1, K2, T, U = C5.shape
    out, R = np.empty(B), np.empty_like(C5)
    lib().orc_jeanie_forward(_p(C5), B, K1, K2, T, U, int(s1), int(s2), float(gamma),
                             _p(out), _p(R))
    return out, R


def jeanie_dp_grad(C5, s1, s2, gamma, g_out, g_R=None):
    """dC of sum(g_out * out) + <g_R, R> (jeanie/_torch_dp.py:41-75)."""
    C5 = _c(C5)
    B, K1, K2, T, U = C5.shape
    _, R = jeanie_dp(C5, s1, s2, gamma)
    g_out = _c(np.broadcast_to(g_out, (B,)))
    gR = None if g_R is None else _c(g_R)
    dC = np.empty_like(C5)
    lib().orc_jeanie_backward(_p(C5), _p(R), _p(g_out), _p(gR), B, K1, K2, T, U, int(s1),
                              int(s2), float(gamma), _p(dC))
    return dC


def optimal_path(D, max_shift=0, start_view=None):
    """Hard (gamma -> 0) path of a [K,T,U] cost (paths.py:85-117)."""
    D = _c(D)
    K, T, U = D.shape
    buf = np.empty(3 * (T + U + 2), dtype=np.int32)
    n = lib().orc_optimal_path(_p(D), K, T, U, int(max_shift),
                               -1 if start_view is None else int(start_view),
                               buf.ctypes.data_as(_ip))
    return [tuple(int(v) for v in buf[3 * i:3 * i + 3]) for i in range(n)]


# ------------------------------------------------------------ cost builders

def _sq_parts(Xf, Yf):
    """GEMM-form squared distance parts (udtw/_autograd.py:19-29)."""
    G = Xf @ np.swapaxes(Yf, -1, -2)
    x2 = (Xf * Xf).sum(-1)
    y2 = (Yf * Yf).sum(-1)
    sq_raw = x2[..., :, None] + y2[..., None, :] - 2.0 * G
    return sq_raw


def udtw_matrices(X, Y, vx, vy, beta, eps):
    """Eqs. (8), (16) in GEMM form: (cost, penalty, sq_raw, var_raw, var)."""
    sq_raw = _sq_parts(X, Y)
    var_raw = 0.5 * (vx[:, :, None] + vy[:, None, :])
    var = np.maximum(var_raw, eps)
    cost = np.maximum(sq_raw, 0.0) / var
    return cost, beta * np.log(var), sq_raw, var_raw, var


# ------------------------------------------------------------- public API

def _udtw_pair(X, Y, sx, sy, beta, gamma, band, eps, g_d, g_p):
    """One uDTW call (udtw/functional.py:147-163 + udtw/_ops.py:186-211):
    values and gradients w.r.t. X, Y, sigma_x, sigma_y."""
    swap = X.shape[1] > Y.shape[1]
    if swap:
        X, Y, sx, sy = Y, X, sy, sx
    vx, vy = sx[..., 0] ** 2, sy[..., 0] ** 2
    cost, pen, sq_raw, var_raw, var = udtw_matrices(X, Y, vx, vy, beta, eps)
    d, p, _, _ = udtw_dp(cost, pen, gamma, band)
    dC, dQ = udtw_dp_grad(cost, pen, gamma, band, g_d, g_p)
    dsq = np.where(sq_raw > 0, dC / var, 0.0)
    dvar = np.where(var_raw > eps, (beta * dQ - dC * cost) / var, 0.0)
    dG = -2.0 * dsq
    dX = dG @ Y + 2.0 * X * dsq.sum(2)[..., None]
    dY = np.swapaxes(dG, 1, 2) @ X + 2.0 * Y * dsq.sum(1)[..., None]
    dsx = (2.0 * sx[..., 0] * 0.5 * dvar.sum(2))[..., None]
    dsy = (2.0 * sy[..., 0] * 0.5 * dvar.sum(1))[..., None]
    if swap:
        dX, dY, dsx, dsy = dY, dX, dsy, dsx
    return d, p, dX, dY, dsx, dsy


def udtw(X, Y, sx, sy, *, beta=1.0, gamma=1.0, normalize=False, bandwidth=None, eps=1e-8,
         g_d=1.0, g_p=0.0):
    """uDTW (udtw/functional.py:166-209): (d, p, dX, dY, dsx, dsy) for the
    loss sum(g_d * d + g_p * p)."""
    X, Y, sx, sy = map(_c, (X, Y, sx, sy))
    band = 0.0 if bandwidth is None else float(bandwidth)
    B = X.shape[0]
    g_d = np.broadcast_to(np.asarray(g_d, dtype=np.float64), (B,)).copy()
    g_p = np.broadcast_to(np.asarray(g_p, dtype=np.float64), (B,)).copy()
    d, p, dX, dY, dsx, dsy = _udtw_pair(X, Y, sx, sy, beta, gamma, band, eps, g_d, g_p)
    if not normalize:
        return d, p, dX, dY, dsx, dsy
    dxx, pxx, a1, a2, a3, a4 = _udtw_pair(X, X, sx, sx, beta, gamma, band, eps,
                                          -0.5 * g_d, -0.5 * g_p)
    dyy, pyy, b1, b2, b3, b4 = _udtw_pair(Y, Y, sy, sy, beta, gamma, band, eps,
                                          -0.5 * g_d, -0.5 * g_p)
    return (d - 0.5 * (dxx + dyy), p - 0.5 * (pxx + pyy),
            dX + a1 + a2, dY + b1 + b2, dsx + a3 + a4, dsy + b3 + b4)


def udtw_from_cost(cost, pen, *, gamma=1.0, bandwidth=None, g_d=1.0, g_p=0.0):
    """uDTW on matrices (udtw/functional.py:104-144): (d, p, dcost, dpen)."""
    band = 0.0 if bandwidth is None else float(bandwidth)
    cost, pen = _c(cost), _c(pen)
    d, p, _, _ = udtw_dp(cost, pen, gamma, band)
    dC, dQ = udtw_dp_grad(cost, pen, gamma, band, g_d, g_p)
    return d, p, dC, dQ


def soft_dtw_from_cost(cost, *, gamma=1.0, bandwidth=None, g=1.0):
    """soft-DTW on a cost [B,T,U] (sdtw.py:29-47): (d, dcost)."""
    d, _, dC, _ = udtw_from_cost(cost, np.zeros_like(cost), gamma=gamma,
                                 bandwidth=bandwidth, g_d=g)
    return d, dC


def soft_dtw(X, Y, *, gamma=1.0, normalize=False, bandwidth=None, g=1.0):
    """soft-DTW on features (sdtw.py:50-92): uDTW with sigma = 1, beta = 0.
    Returns (d, dX, dY)."""
    X, Y = _c(X), _c(Y)
    ones_x = np.ones(X.shape[:2] + (1,))
    ones_y = np.ones(Y.shape[:2] + (1,))
    d, _, dX, dY, _, _ = udtw(X, Y, ones_x, ones_y, beta=0.0, gamma=gamma, normalize=normalize,
                              bandwidth=bandwidth, g_d=g, g_p=0.0)
    return d, dX, dY


def _shifts(max_shift, axes):
    s = (max_shift,) * axes if isinstance(max_shift, int) else tuple(int(m) for m in max_shift)
    return s + (0,) * (2 - axes)


def jeanie_from_cost(cost, *, gamma=0.1, max_shift=1, g=1.0, g_R=None):
    """JEANIE on [B,K,T,U] or [B,K1,K2,T,U] (jeanie/functional.py:28-61, 171-193).
    Returns (d, R, dcost) with R and dcost shaped like cost."""
    cost = _c(cost)
    one = cost.ndim == 4
    s1, s2 = _shifts(max_shift, 1 if one else 2)
    c5 = cost[:, :, None] if one else cost
    s1, s2 = min(s1, c5.shape[1] - 1), min(s2, c5.shape[2] - 1)
    gR5 = None if g_R is None else (_c(g_R)[:, :, None] if one else _c(g_R))
    d, R = jeanie_dp(c5, s1, s2, gamma)
    dC = jeanie_dp_grad(c5, s1, s2, gamma, g, gR5)
    if one:
        R, dC = R[:, :, 0], dC[:, :, 0]
    return d, R, dC


def sq_euclidean_cost(q, s):
    """squared_euclidean_cost (jeanie/distances.py:25-31) and its raw value."""
    sb = s[..., None, :, :] if q.ndim > s.ndim else s
    q2 = (q * q).sum(-1)[..., :, None]
    s2 = (sb * sb).sum(-1)[..., None, :]
    raw = q2 + s2 - 2.0 * (q @ np.swapaxes(sb, -1, -2))
    return np.maximum(raw, 0.0), raw


def distance(name, q, s, g=None):
    """Base distances of jeanie/distances.py:25-51 and their gradients w.r.t.
    (q, s) for the cotangent g (default ones)."""
    q, s = _c(q), _c(s)
    bcast = q.ndim > s.ndim
    sb = s[..., None, :, :] if bcast else s
    if name == "rbf_cost":
        diff = q[..., :, None, :] - sb[..., None, :, :]
        e = np.exp(-0.5 * diff ** 2)
        val = (2.0 - 2.0 * e).sum(-1)
        gg = np.ones_like(val) if g is None else g
        dd = gg[..., None] * 2.0 * e * 0.5 * 2.0 * diff
        dq = dd.sum(-2)
        ds = -dd.sum(-3)
    else:
        sq, raw = sq_euclidean_cost(q, s)
        gg = np.ones_like(sq) if g is None else g
        if name == "euclidean_cost":
            pos = raw > 0
            val = np.where(pos, np.sqrt(np.where(pos, sq, 1.0)), 0.0)
            dsq = np.where(pos, 0.5 * gg / np.where(pos, val, 1.0), 0.0)
        else:
            val = sq
            dsq = np.where(raw > 0, gg, 0.0)
        dq = 2.0 * q * dsq.sum(-1)[..., None] - 2.0 * dsq @ sb
        ds = 2.0 * sb * dsq.sum(-2)[..., None] - 2.0 * np.swapaxes(dsq, -1, -2) @ q
    if bcast:
        ds = ds.sum(-3)
    return val, dq, ds


def jeanie(query, support, *, gamma=0.1, max_shift=1, metric="euclidean", g=1.0, g_R=None):
    """JEANIE on features (jeanie/functional.py:64-106, 141-168): returns
    (d, R, dquery, dsupport).  Cost in GEMM form (jeanie/_autograd.py:58-70)."""
    query, support = _c(query), _c(support)
    one = query.ndim == 4
    q5 = query[:, :, None] if one else query
    B, K1, K2, T, D = q5.shape
    U = support.shape[1]
    qf = q5.reshape(B, K1 * K2 * T, D)
    name = {"euclidean": "euclidean_cost", "sqeuclidean": "squared_euclidean_cost",
            "rbf": "rbf_cost"}[metric]
    cost = distance(name, qf, support)[0].reshape(B, K1, K2, T, U)
    c_in = cost[:, :, 0] if one else cost
    d, R, dC = jeanie_from_cost(c_in, gamma=gamma, max_shift=max_shift, g=g, g_R=g_R)
    dC5 = dC[:, :, None] if one else dC
    _, dq, ds = distance(name, qf, support, g=dC5.reshape(B, K1 * K2 * T, U))
    dq = dq.reshape(query.shape)
    return d, R, dq, ds


def fvm_from_cost(cost, *, gamma=0.1, g=1.0):
    """FVM on a cost [B, K..., T, U] (jeanie/fvm.py:15-38): (d, dcost)."""
    cost = _c(cost)
    B, T, U = cost.shape[0], cost.shape[-2], cost.shape[-1]
    flat = cost.reshape(B, -1, T, U)
    m = flat.min(1, keepdims=True)
    e = np.exp((m - flat) / gamma)
    temporal = m[:, 0] - gamma * np.log(e.sum(1))
    d, dT = soft_dtw_from_cost(temporal, gamma=gamma, g=g)
    w = e / e.sum(1, keepdims=True)
    return d, (w * dT[:, None]).reshape(cost.shape)


def fvm(query, support, *, gamma=0.1, metric="euclidean", g=1.0):
    """FVM on features (jeanie/fvm.py:41-67): (d, dquery, dsupport)."""
    query, support = _c(query), _c(support)
    B, T, D = query.shape[0], query.shape[-2], query.shape[-1]
    U = support.shape[-2]
    name = {"euclidean": "euclidean_cost", "sqeuclidean": "squared_euclidean_cost",
            "rbf": "rbf_cost"}[metric]
    q = query.reshape(B, -1, T, D)
    if support.ndim == 3:
        cost, _, _ = distance(name, q, support)
        d, dcost = fvm_from_cost(cost, gamma=gamma, g=g)
        _, dq, ds = distance(name, q, support, g=dcost)
    else:
        s = support.reshape(B, -1, U, D)
        Kq, Ks = q.shape[1], s.shape[1]
        qq = np.broadcast_to(q[:, :, None], (B, Kq, Ks, T, D))
        ss = np.broadcast_to(s[:, None], (B, Kq, Ks, U, D))
        cost, _, _ = distance(name, qq, ss)
        d, dcost = fvm_from_cost(cost, gamma=gamma, g=g)
        _, dqq, dss = distance(name, qq, ss, g=dcost)
        dq, ds = dqq.sum(2), dss.sum(1).reshape(support.shape)
    return d, dq.reshape(query.shape), ds
