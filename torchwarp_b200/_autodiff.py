"""Differentiable restatements of the soft-min recurrences in torch operations,
used only for derivatives beyond the first order.

First-order values (reverse and forward mode) always come from the native
kernels.  When a gradient is itself differentiated (create_graph=True, MAML
meta-gradients, torch.func.hessian = jacfwd(jacrev), third derivatives), the
native first-order backward is wrapped in ``FirstOrder``: its forward is the
native call, and its own backward and jvp are taken by torch.func through the
functions below, which compute the same quantities with differentiable torch
operations on the GPU.  The reference routes every order beyond the first the
same way, through its pure-PyTorch dynamic programs
(hibana2077/torchwarp src/torchwarp/udtw/_ops.py:226-258, udtw/_autograd.py,
jeanie/_autograd.py).

The DPs run over anti-diagonals: every cell of a diagonal at once, the
diagonal's predecessors gathered from the two diagonals before it.
Unreachable predecessors carry a large finite value (so no inf - inf enters
a log-sum-exp or its derivatives) and contribute a zero weight.
"""

import torch
import torch.nn.functional as F

BIG = 1e30


# ------------------------------------------------------------ soft-DTW / uDTW

def udtw_dp(cost, penalty, gamma, bandwidth=0.0):
    """(distance [B], penalty sum [B]) of the uDTW recurrence on cost and
    penalty [B, N, M] (penalty None: soft-DTW, penalty sum 0).
    R_ij = C_ij + softmin_gamma(R_i-1,j-1, R_i-1,j, R_i,j-1), R_-1,-1 = 0;
    P_ij = Q_ij + sum_p softmax_p P_p (udtw/_torch_dp.py:14-42); cells outside
    the Sakoe-Chiba band |i - j| <= bandwidth (bandwidth > 0) are unreachable."""
    B, N, M = cost.shape
    dev = cost.device
    rows = torch.arange(N, device=dev)
    big = cost.new_full((B, 1), BIG)
    zero = cost.new_zeros((B, 1))
    # diagonal values indexed by row i + 1 (index 0 is row -1)
    r1 = r2 = None
    p1 = p2 = None
    for d in range(N + M - 1):
        cols = d - rows
        ok = (cols >= 0) & (cols < M)
        if bandwidth > 0:
            ok = ok & ((rows - cols).abs() <= bandwidth)
        cj = cols.clamp(0, M - 1)
        c = cost[:, rows, cj]
        q = penalty[:, rows, cj] if penalty is not None else None
        if d == 0:
            r = torch.where(ok, c, BIG)
            p = torch.where(ok, q, 0.0) if q is not None else None
        else:
            diag = r2[:, :-1] if r2 is not None else None
            up, left = r1[:, :-1], r1[:, 1:]
            if diag is None:   # d == 1: the diagonal predecessor is row -1
                diag = big.expand(B, N)
            cand = torch.stack((diag, up, left), 1)          # [B, 3, N]
            z = -cand / gamma
            r = c - gamma * torch.logsumexp(z, 1)
            reach = ok & (r < 0.5 * BIG)
            r = torch.where(reach, r, BIG)
            if q is not None:
                pdiag = p2[:, :-1] if p2 is not None else zero.expand(B, N)
                pc = torch.stack((pdiag, p1[:, :-1], p1[:, 1:]), 1)
                p = torch.where(reach, q + (torch.softmax(z, 1) * pc).sum(1), 0.0)
            else:
                p = None
        r2, r1 = r1, torch.cat((big, r), 1)
        if q is not None:
            p2, p1 = p1, torch.cat((zero, p), 1)
    dist = r1[:, N]
    pen = p1[:, N] if penalty is not None else cost.new_zeros(B)
    return dist, pen


def sq_euclid(X, Y):
    """max(|x_i|^2 + |y_j|^2 - 2 x_i.y_j, 0), the GEMM form of the kernels."""
    x2 = (X * X).sum(-1)
    y2 = (Y * Y).sum(-1)
    return (x2[..., :, None] + y2[..., None, :] - 2.0 * X @ Y.transpose(-1, -2)).clamp_min(0)


def euclid(X, Y):
    """sqrt of sq_euclid with zero gradient at 0 (jeanie/distances.py:34-38)."""
    sq = sq_euclid(X, Y)
    pos = sq > 0
    return torch.where(pos, torch.sqrt(torch.where(pos, sq, torch.ones_like(sq))),
                       torch.zeros_like(sq))


def rbf(X, Y, sigma):
    diff = X[..., :, None, :] - Y[..., None, :, :]
    return (2.0 - 2.0 * torch.exp(-sigma * diff * diff)).sum(-1)


def udtw_matrices(X, Y, vx, vy, beta, eps):
    """(cost, penalty) of uDTW Eqs. 8 and 16; vx, vy [B, N], [B, M] variances."""
    sq = sq_euclid(X, Y)
    var = (0.5 * (vx[:, :, None] + vy[:, None, :])).clamp_min(eps)
    return sq / var, beta * torch.log(var)


# ------------------------------------------------------------------ JEANIE

def _window(x, s1, s2):
    """x [B, K1, K2, n] -> [B, K1, K2, n, W]: every viewpoint's window
    |n1' - n1| <= s1, |n2' - n2| <= s2 (padded with BIG)."""
    B, K1, K2, n = x.shape
    y = x.permute(0, 3, 1, 2)                                  # [B, n, K1, K2]
    y = F.pad(y, (s2, s2, s1, s1), value=BIG)
    y = y.unfold(2, 2 * s1 + 1, 1).unfold(3, 2 * s2 + 1, 1)    # [B, n, K1, K2, w1, w2]
    return y.reshape(B, n, K1, K2, -1).permute(0, 2, 3, 1, 4)


def jeanie_dp(cost5, s1, s2, gamma):
    """(out [B], R [B, K1, K2, T, U]) of JEANIE on a cost [B, K1, K2, T, U]
    (jeanie/_torch_dp.py:14-38): R = C + softmin over the viewpoint window of
    the three temporal predecessors; out = softmin over viewpoints of the end
    cells."""
    B, K1, K2, T, U = cost5.shape
    dev = cost5.device
    cells = [None] * (T * U)
    diags = []          # per diagonal: (tlo, values [B, K1, K2, nt])
    for d in range(T + U - 1):
        tlo, thi = max(0, d - U + 1), min(T - 1, d)
        ts = torch.arange(tlo, thi + 1, device=dev)
        us = d - ts
        c = cost5[:, :, :, ts, us]                            # [B, K1, K2, nt]
        if d == 0:
            r = c
        else:
            def pred(dd, dt, du):
                # values of cells (t + dt, u + du) from diagonal dd, BIG when absent
                p_lo, pv = diags[dd]
                tt = ts + dt
                uu = us + du
                p_hi = p_lo + pv.shape[-1] - 1
                okp = (tt >= p_lo) & (tt <= p_hi) & (uu >= 0) & (uu < U) & (tt >= 0)
                idx = (tt - p_lo).clamp(0, pv.shape[-1] - 1)
                v = pv[..., idx]
                return torch.where(okp, v, BIG)
            cand = torch.cat((_window(pred(d - 1, -1, 0), s1, s2),
                              _window(pred(d - 1, 0, -1), s1, s2),
                              (_window(pred(d - 2, -1, -1), s1, s2) if d >= 2 else
                               torch.full_like(_window(c, s1, s2), BIG))), -1)
            r = c - gamma * torch.logsumexp(-cand / gamma, -1)
        diags.append((tlo, r))
        for k, t in enumerate(range(tlo, thi + 1)):
            cells[t * U + (d - t)] = r[..., k]
    R = torch.stack(cells, -1).reshape(B, K1, K2, T, U)
    end = R[..., T - 1, U - 1].reshape(B, K1 * K2)
    out = -gamma * torch.logsumexp(-end / gamma, 1)
    return out, R


def viewpoint_softmin(cost, gamma):
    """[B, Kf, T, U] -> [B, T, U]: -gamma logsumexp_n(-cost / gamma)
    (jeanie/fvm.py:36-37)."""
    return -gamma * torch.logsumexp(-cost / gamma, 1)


def qs_cost(query, support, metric, sigma=None):
    """Query/support cost [B, R, U] from [B, R, D] x [B, U, D]: metric 0
    squared Euclidean, 1 Euclidean, None with sigma: rbf."""
    if sigma is not None:
        return rbf(query, support, sigma)
    return euclid(query, support) if metric == 1 else sq_euclid(query, support)


# ----------------------------------------------- first order, all orders above

def first_order_of(fn, n_primal):
    """(primals..., cotangents...) -> vjp of fn at the primals, itself
    differentiable: the first-order gradient as a differentiable function."""
    def g(*args):
        primals, cots = args[:n_primal], args[n_primal:]
        _, pull = torch.func.vjp(fn, *primals)
        return pull(tuple(cots) if len(cots) > 1 else cots[0])
    return g


class FirstOrder(torch.autograd.Function):
    """A native first-order backward whose own derivatives (reverse and
    forward mode) go through torch.func on ``ref``, a differentiable function
    computing the same gradients.

    apply(native, ref, n_const, *args): ``native(*args)`` returns the
    gradients (a tuple) from the native kernels; ``ref(*args)`` returns the
    same tuple with differentiable torch operations.  The first ``n_const``
    args are constants both functions read but nothing differentiates (a
    saved stream, for one); the rest are the tensors the gradients depend on
    (primal inputs, then the incoming cotangents), None allowed.  Both
    functions take the tensors as arguments, so vmap levels stay apart."""

    generate_vmap_rule = True

    @staticmethod
    def forward(native, ref, n_const, *args):
        return tuple(native(*args))

    @staticmethod
    def setup_context(ctx, inputs, output):
        native, ref, n_const, *args = inputs
        ctx.ref = ref
        ctx.n_const = n_const
        ctx.none = [a is None for a in args]
        kept = [a for a in args if a is not None]
        ctx.save_for_backward(*kept)
        ctx.save_for_forward(*kept)

    @staticmethod
    def _split(ctx):
        it = iter(ctx.saved_tensors)
        args = [None if n else next(it) for n in ctx.none]
        live = [i for i, a in enumerate(args)
                if i >= ctx.n_const and a is not None and a.is_floating_point()]

        def f(*xs):
            full = list(args)
            for i, x in zip(live, xs):
                full[i] = x
            return tuple(ctx.ref(*full))

        return args, live, f

    @staticmethod
    def backward(ctx, *gouts):
        args, live, f = FirstOrder._split(ctx)
        outs, pull = torch.func.vjp(f, *[args[i] for i in live])
        cots = tuple(torch.zeros_like(o) if g is None else g for o, g in zip(outs, gouts))
        grads = pull(cots)
        res = [None] * len(args)
        for i, g in zip(live, grads):
            res[i] = g
        return (None, None, None) + tuple(res)

    @staticmethod
    def jvp(ctx, _native_t, _ref_t, _n_t, *tangents):
        args, live, f = FirstOrder._split(ctx)
        prim = tuple(args[i].contiguous() for i in live)
        tans = tuple((torch.zeros_like(args[i]) if tangents[i] is None
                      else tangents[i].contiguous()) for i in live)
        return torch.func.jvp(f, prim, tans)[1]


def first_order(native, ref, n_const, *args):
    """The native first-order gradients, differentiable through ``ref``."""
    return FirstOrder.apply(native, ref, n_const, *args)
