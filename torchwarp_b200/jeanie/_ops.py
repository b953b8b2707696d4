"""JEANIE, FVM and the query/support cost as torch custom operators over the C ABI.

Mirrors the reference op layer (hibana2077/torchwarp src/torchwarp/jeanie/_ops.py:
``dp``/``dp_backward`` :110-139, ``features``/``features_backward`` :155-230,
autograd Functions :299-447) with native sm_100a kernels only:

* ``torchwarp_b200::jeanie_dp(cost5, s1, s2, gamma)`` -> (out [B], R): the
  DP on a [B, K1, K2, T, U] cost; R (natural layout) is both the saved state
  and the differentiable accumulator.
* ``torchwarp_b200::jeanie_dp_backward(cost5, R, grad_out, grad_R?, ...)``.
* ``torchwarp_b200::qs_cost(query, support, metric)`` -> cost [B, R, U] and
  its backward, the (squared) Euclidean query/support cost that replaces the
  reference's bmm + relayout + fused kernel cost.
* ``torchwarp_b200::fvm_softmin(cost, gamma)`` -> temporal [B, T, U] and its
  backward (FVM's viewpoint soft-min).

Each op has a fake implementation (torch.compile), a vmap rule that merges
the vmapped dimension with the pairs (``torchwarp_b200._vmap``), and runs in
float32 under autocast; the autograd Functions let torch.func generate their
vmap rules from these.  The backward ops are first-order only.
"""

import os
from typing import Optional, Tuple

import torch
from torch import Tensor

from .. import _native as nat
from .. import _autodiff as AD
from .. import _transforms
from .._vmap import register_fold_rule, round_to_pairs


def _register_autocast(op):
    for device in ("cuda", "cpu"):
        torch.library.register_autocast(op, device, torch.float32)


def _fn(name, dtype):
    return getattr(nat.lib(), name + "_" + nat.suffix(dtype))


# ------------------------------------------------------------ JEANIE DP

@torch.library.custom_op("torchwarp_b200::jeanie_dp", mutates_args=())
def jeanie_dp(cost: Tensor, s1: int, s2: int, gamma: float) -> Tuple[Tensor, Tensor]:
    nat.require_cuda(cost)
    B, K1, K2, T, U = cost.shape
    cost = cost.contiguous()
    out = cost.new_empty(B)
    R = torch.empty_like(cost)
    if B:
        with torch.cuda.device(cost.device):
            nat.check(nat.call("jeanie_forward", _fn("tw_jeanie_forward", cost.dtype),
                               nat.ptr(cost), B, K1, K2, T, U, int(s1), int(s2), float(gamma),
                               nat.ptr(out), nat.ptr(R), nat.stream_of(cost)), "tw_jeanie_forward")
    return out, R


@jeanie_dp.register_fake
def _(cost, s1, s2, gamma):
    return cost.new_empty(cost.shape[0]), torch.empty_like(cost)


@torch.library.custom_op("torchwarp_b200::jeanie_dp_backward", mutates_args=())
def jeanie_dp_backward(cost: Tensor, R: Tensor, grad_out: Tensor, grad_R: Optional[Tensor], s1: int,
                       s2: int, gamma: float) -> Tensor:
    nat.require_cuda(cost)
    B, K1, K2, T, U = cost.shape
    cost, R = cost.contiguous(), R.contiguous()
    grad_out = grad_out.to(cost.dtype).contiguous()
    gR = None if grad_R is None else grad_R.to(cost.dtype).contiguous()
    d_cost = torch.empty_like(cost)
    if B:
        with torch.cuda.device(cost.device):
            nat.check(nat.call("jeanie_backward", _fn("tw_jeanie_backward", cost.dtype),
                               nat.ptr(cost), nat.ptr(R), nat.ptr(grad_out), nat.ptr(gR), B, K1,
                               K2, T, U, int(s1), int(s2), float(gamma), nat.ptr(d_cost),
                               nat.stream_of(cost)), "tw_jeanie_backward")
    return d_cost


@jeanie_dp_backward.register_fake
def _(cost, R, grad_out, grad_R, s1, s2, gamma):
    return torch.empty_like(cost)


_register_autocast(jeanie_dp)
_register_autocast(jeanie_dp_backward)
register_fold_rule(jeanie_dp)
register_fold_rule(jeanie_dp_backward)


class JeanieDP(torch.autograd.Function):
    """cost5 -> (out, R).  R (the accumulator) is differentiable when the
    caller asked for it (keep_R), and an internal, non-differentiable output
    otherwise.

    Forward mode: the tangent of the distance along T is <dout/dcost, T>, from
    one native backward with unit seeds; with the accumulator requested, the
    tangents of both outputs come from torch.func.jvp of the differentiable
    restatement of the DP.  Differentiating the backward again goes through
    the same restatement (native first-order values)."""

    generate_vmap_rule = True

    @staticmethod
    def forward(cost, s1, s2, gamma, keep_R):
        return jeanie_dp(cost, s1, s2, gamma)

    @staticmethod
    def setup_context(ctx, inputs, output):
        cost, s1, s2, gamma, keep_R = inputs
        ctx.set_materialize_grads(False)
        if not keep_R:
            ctx.mark_non_differentiable(output[1])
        ctx.save_for_backward(cost, output[1])
        ctx.save_for_forward(cost, output[1])
        ctx.args = (s1, s2, gamma, keep_R)

    @staticmethod
    def backward(ctx, g_out, g_R):
        cost, R = ctx.saved_tensors
        s1, s2, gamma, _ = ctx.args
        if g_out is None:
            g_out = cost.new_zeros(cost.shape[0])
        if torch.is_grad_enabled():
            d_cost, = AD.first_order(_jeanie_grad_native(s1, s2, gamma),
                                     _jeanie_grad_ref(s1, s2, gamma), 1, R, cost, g_out, g_R)
            return d_cost, None, None, None, None
        return JeanieDP._backward_once(ctx, cost, R, g_out, g_R)

    @staticmethod
    @_transforms.once_differentiable
    def _backward_once(ctx, cost, R, g_out, g_R):
        s1, s2, gamma, _ = ctx.args
        return jeanie_dp_backward(cost, R, g_out, g_R, s1, s2, gamma), None, None, None, None

    @staticmethod
    def jvp(ctx, cost_t, _s1_t, _s2_t, _gamma_t, _keep_t):
        cost, R = ctx.saved_tensors
        s1, s2, gamma, keep_R = ctx.args
        if keep_R:
            ct = torch.zeros_like(cost) if cost_t is None else cost_t.to(cost.dtype)
            return torch.func.jvp(lambda c: AD.jeanie_dp(c, s1, s2, gamma),
                                  (cost.contiguous(),), (ct.contiguous(),))[1]
        B = cost.shape[0]
        if cost_t is None:
            return cost.new_zeros(B), None
        w = jeanie_dp_backward(cost, R, cost.new_ones(B), None, s1, s2, gamma)
        return (w * cost_t).flatten(1).sum(1), None


def _jeanie_grad_native(s1, s2, gamma):
    """(R, cost, g_out, g_R) -> (d_cost,), native."""
    def f(R, cost, g_out, g_R):
        return (jeanie_dp_backward(cost, R, g_out, g_R, s1, s2, gamma),)
    return f


def _jeanie_grad_ref(s1, s2, gamma):
    """(R, cost, g_out, g_R) -> (d_cost,), differentiable."""
    def f(R, cost, g_out, g_R):
        _, pull = torch.func.vjp(lambda c: AD.jeanie_dp(c, s1, s2, gamma), cost)
        return pull((g_out, torch.zeros_like(cost) if g_R is None else g_R))
    return f


# ------------------------------------------------------ query/support cost

@torch.library.custom_op("torchwarp_b200::qs_cost", mutates_args=())
def qs_cost(query: Tensor, support: Tensor, metric: int) -> Tensor:
    nat.require_cuda(query, support)
    B, Rr, D = query.shape
    U = support.shape[1]
    query, support = query.contiguous(), support.contiguous()
    cost = query.new_empty(B, Rr, U)
    if B and Rr and U:
        with torch.cuda.device(query.device):
            nat.check(nat.call("qs_cost", _fn("tw_qs_cost", query.dtype), nat.ptr(query),
                               nat.ptr(support), B, Rr, U, D, int(metric), nat.ptr(cost),
                               nat.stream_of(query)), "tw_qs_cost")
    return cost


@qs_cost.register_fake
def _(query, support, metric):
    return query.new_empty(query.shape[0], query.shape[1], support.shape[1])


@torch.library.custom_op("torchwarp_b200::qs_cost_backward", mutates_args=())
def qs_cost_backward(query: Tensor, support: Tensor, cost: Tensor, d_cost: Tensor,
                     metric: int) -> Tuple[Tensor, Tensor]:
    nat.require_cuda(query, support)
    B, Rr, D = query.shape
    U = support.shape[1]
    query, support, cost = query.contiguous(), support.contiguous(), cost.contiguous()
    d_cost = d_cost.to(query.dtype).contiguous()
    dq, ds = torch.empty_like(query), torch.empty_like(support)
    if B and Rr and U:
        with torch.cuda.device(query.device):
            nat.check(nat.call("qs_cost_grad", _fn("tw_qs_cost_grad", query.dtype),
                               nat.ptr(query), nat.ptr(support), nat.ptr(cost), nat.ptr(d_cost),
                               B, Rr, U, D, int(metric), nat.ptr(dq), nat.ptr(ds),
                               nat.stream_of(query)), "tw_qs_cost_grad")
    return dq, ds


@qs_cost_backward.register_fake
def _(query, support, cost, d_cost, metric):
    return torch.empty_like(query), torch.empty_like(support)


_register_autocast(qs_cost)
_register_autocast(qs_cost_backward)
register_fold_rule(qs_cost)
register_fold_rule(qs_cost_backward)


class QSCost(torch.autograd.Function):
    """(query [B,R,D], support [B,U,D]) -> cost [B,R,U]."""

    generate_vmap_rule = True

    @staticmethod
    def forward(query, support, metric):
        return qs_cost(query, support, metric)

    @staticmethod
    def setup_context(ctx, inputs, output):
        query, support, metric = inputs
        ctx.save_for_backward(query, support, output)
        ctx.save_for_forward(query, support, output)
        ctx.metric = metric

    @staticmethod
    def backward(ctx, g):
        query, support, cost = ctx.saved_tensors
        if torch.is_grad_enabled():
            metric = ctx.metric

            def native(cost_, q, s_, g_):
                return qs_cost_backward(q, s_, cost_, g_, metric)

            def ref(cost_, q, s_, g_):
                _, pull = torch.func.vjp(lambda a, b: AD.qs_cost(a, b, metric), q, s_)
                return pull(g_)

            dq, ds = AD.first_order(native, ref, 1, cost, query, support, g)
            return dq, ds, None
        return QSCost._backward_once(ctx, query, support, cost, g)

    @staticmethod
    @_transforms.once_differentiable
    def _backward_once(ctx, query, support, cost, g):
        dq, ds = qs_cost_backward(query, support, cost, g, ctx.metric)
        return dq, ds, None

    @staticmethod
    def jvp(ctx, q_t, s_t, _metric_t):
        """Tangent of the cost: sq' = 2 q.q' + 2 s.s' - 2 (q' s^T + q s'^T), zero
        where the clamp holds sq at 0; the Euclidean root divides by 2 cost."""
        q, s, cost = ctx.saved_tensors
        q_t = torch.zeros_like(q) if q_t is None else q_t.to(q.dtype)
        s_t = torch.zeros_like(s) if s_t is None else s_t.to(s.dtype)
        sq_t = (2.0 * (q * q_t).sum(-1)[:, :, None] + 2.0 * (s * s_t).sum(-1)[:, None, :]
                - 2.0 * (torch.bmm(q_t, s.transpose(1, 2)) + torch.bmm(q, s_t.transpose(1, 2))))
        pos = cost > 0
        if ctx.metric == 1:
            sq_t = sq_t / (2.0 * torch.where(pos, cost, torch.ones_like(cost)))
        return torch.where(pos, sq_t, torch.zeros_like(sq_t))


# ------------------------------------------------------------ rbf cost

@torch.library.custom_op("torchwarp_b200::qs_rbf_cost", mutates_args=())
def qs_rbf_cost(query: Tensor, support: Tensor, sigma: float) -> Tensor:
    """cost [B,R,U] = sum_d [2 - 2 exp(-sigma (q - s)^2)], without the
    [B,R,U,D] difference tensor (jeanie/distances.py:41-51)."""
    nat.require_cuda(query, support)
    B, Rr, D = query.shape
    U = support.shape[1]
    query, support = query.contiguous(), support.contiguous()
    cost = query.new_empty(B, Rr, U)
    if B and Rr and U:
        with torch.cuda.device(query.device):
            nat.check(nat.call("qs_rbf_cost", _fn("tw_qs_rbf_cost", query.dtype),
                               nat.ptr(query), nat.ptr(support), B, Rr, U, D, float(sigma),
                               nat.ptr(cost), nat.stream_of(query)), "tw_qs_rbf_cost")
    return cost


@qs_rbf_cost.register_fake
def _(query, support, sigma):
    return query.new_empty(query.shape[0], query.shape[1], support.shape[1])


@torch.library.custom_op("torchwarp_b200::qs_rbf_cost_backward", mutates_args=())
def qs_rbf_cost_backward(query: Tensor, support: Tensor, d_cost: Tensor,
                         sigma: float) -> Tuple[Tensor, Tensor]:
    nat.require_cuda(query, support)
    B, Rr, D = query.shape
    U = support.shape[1]
    query, support = query.contiguous(), support.contiguous()
    d_cost = d_cost.to(query.dtype).contiguous()
    dq, ds = torch.empty_like(query), torch.empty_like(support)
    if B and Rr and U:
        with torch.cuda.device(query.device):
            nat.check(nat.call("qs_rbf_cost_grad", _fn("tw_qs_rbf_cost_grad", query.dtype),
                               nat.ptr(query), nat.ptr(support), nat.ptr(d_cost), B, Rr, U, D,
                               float(sigma), nat.ptr(dq), nat.ptr(ds), nat.stream_of(query)),
                      "tw_qs_rbf_cost_grad")
    elif B:
        dq.zero_()
        ds.zero_()
    return dq, ds


@qs_rbf_cost_backward.register_fake
def _(query, support, d_cost, sigma):
    return torch.empty_like(query), torch.empty_like(support)


_register_autocast(qs_rbf_cost)
_register_autocast(qs_rbf_cost_backward)
register_fold_rule(qs_rbf_cost)
register_fold_rule(qs_rbf_cost_backward)


class QSRbfCost(torch.autograd.Function):
    """(query [B,R,D], support [B,U,D]) -> rbf cost [B,R,U]."""

    generate_vmap_rule = True

    @staticmethod
    def forward(query, support, sigma):
        return qs_rbf_cost(query, support, sigma)

    @staticmethod
    def setup_context(ctx, inputs, output):
        query, support, sigma = inputs
        ctx.save_for_backward(query, support)
        ctx.save_for_forward(query, support)
        ctx.sigma = sigma

    @staticmethod
    def backward(ctx, g):
        query, support = ctx.saved_tensors
        if torch.is_grad_enabled():
            sigma = ctx.sigma

            def native(q, s_, g_):
                return qs_rbf_cost_backward(q, s_, g_, sigma)

            def ref(q, s_, g_):
                _, pull = torch.func.vjp(lambda a, b: AD.rbf(a, b, sigma), q, s_)
                return pull(g_)

            dq, ds = AD.first_order(native, ref, 0, query, support, g)
            return dq, ds, None
        return QSRbfCost._backward_once(ctx, query, support, g)

    @staticmethod
    @_transforms.once_differentiable
    def _backward_once(ctx, query, support, g):
        dq, ds = qs_rbf_cost_backward(query, support, g, ctx.sigma)
        return dq, ds, None

    @staticmethod
    def jvp(ctx, q_t, s_t, _sigma_t):
        query, support = ctx.saved_tensors
        q_t = torch.zeros_like(query) if q_t is None else q_t.to(query.dtype)
        s_t = torch.zeros_like(support) if s_t is None else s_t.to(support.dtype)
        return torch.func.jvp(lambda a, b: AD.rbf(a, b, ctx.sigma),
                              (query.contiguous(), support.contiguous()),
                              (q_t.contiguous(), s_t.contiguous()))[1]


# ------------------------------------------------------------ FVM soft-min

@torch.library.custom_op("torchwarp_b200::fvm_softmin", mutates_args=())
def fvm_softmin(cost: Tensor, gamma: float) -> Tensor:
    nat.require_cuda(cost)
    B, Kf, T, U = cost.shape
    cost = cost.contiguous()
    out = cost.new_empty(B, T, U)
    if B:
        with torch.cuda.device(cost.device):
            nat.check(nat.call("fvm_softmin", _fn("tw_fvm_softmin", cost.dtype), nat.ptr(cost), B,
                               Kf, T * U, float(gamma), nat.ptr(out), nat.stream_of(cost)),
                      "tw_fvm_softmin")
    return out


@fvm_softmin.register_fake
def _(cost, gamma):
    return cost.new_empty(cost.shape[0], cost.shape[2], cost.shape[3])


@torch.library.custom_op("torchwarp_b200::fvm_softmin_backward", mutates_args=())
def fvm_softmin_backward(cost: Tensor, d_temporal: Tensor, gamma: float) -> Tensor:
    nat.require_cuda(cost)
    B, Kf, T, U = cost.shape
    cost = cost.contiguous()
    d_temporal = d_temporal.to(cost.dtype).contiguous()
    d_cost = torch.empty_like(cost)
    if B:
        with torch.cuda.device(cost.device):
            nat.check(nat.call("fvm_softmin_backward", _fn("tw_fvm_softmin_backward", cost.dtype),
                               nat.ptr(cost), nat.ptr(d_temporal), B, Kf, T * U, float(gamma),
                               nat.ptr(d_cost), nat.stream_of(cost)), "tw_fvm_softmin_backward")
    return d_cost


@fvm_softmin_backward.register_fake
def _(cost, d_temporal, gamma):
    return torch.empty_like(cost)


_register_autocast(fvm_softmin)
_register_autocast(fvm_softmin_backward)
register_fold_rule(fvm_softmin)
register_fold_rule(fvm_softmin_backward)


class FvmSoftmin(torch.autograd.Function):
    """cost [B,Kf,T,U] -> temporal [B,T,U]."""

    generate_vmap_rule = True

    @staticmethod
    def forward(cost, gamma):
        return fvm_softmin(cost, gamma)

    @staticmethod
    def setup_context(ctx, inputs, output):
        cost, gamma = inputs
        ctx.save_for_backward(cost)
        ctx.save_for_forward(cost)
        ctx.gamma = gamma

    @staticmethod
    def backward(ctx, g):
        (cost,) = ctx.saved_tensors
        if torch.is_grad_enabled():
            gamma = ctx.gamma

            def native(c, g_):
                return (fvm_softmin_backward(c, g_, gamma),)

            def ref(c, g_):
                _, pull = torch.func.vjp(lambda x: AD.viewpoint_softmin(x, gamma), c)
                return pull(g_)

            d_cost, = AD.first_order(native, ref, 0, cost, g)
            return d_cost, None
        return FvmSoftmin._backward_once(ctx, cost, g)

    @staticmethod
    @_transforms.once_differentiable
    def _backward_once(ctx, cost, g):
        return fvm_softmin_backward(cost, g, ctx.gamma), None

    @staticmethod
    def jvp(ctx, cost_t, _gamma_t):
        """temporal' = sum over viewpoints of softmax weights * cost'; the
        weights come from the native backward with a unit seed."""
        (cost,) = ctx.saved_tensors
        B, Kf, T, U = cost.shape
        if cost_t is None:
            return cost.new_zeros(B, T, U)
        w = fvm_softmin_backward(cost, cost.new_ones(B, T, U), ctx.gamma)
        return (w * cost_t.to(cost.dtype)).sum(1)


JeanieDPTraced = _transforms.traceable(JeanieDP)
QSCostTraced = _transforms.traceable(QSCost)
FvmSoftminTraced = _transforms.traceable(FvmSoftmin)


# ------------------------------------------- fused JEANIE / FVM (float32)

def fused_supported(K, T, U, D, fvm, features):
    """Whether tw_jeanie_fused_* take this shape (features: even D <= 256,
    U <= 15; a pair's state within the kernel's shared memory).  The
    environment variable TW_JEANIE_UNFUSED (any value but "0") turns the
    fused path off, for A/B comparisons with the separate cost / soft-min /
    DP kernels."""
    env = os.environ.get("TW_JEANIE_UNFUSED", "")
    if env not in ("", "0"):
        return False
    return _fused_supported_native(int(K), int(T), int(U), int(D), int(fvm), int(features))


@torch._dynamo.assume_constant_result
def _fused_supported_native(K, T, U, D, fvm, features):
    # a pure function of its integer arguments: under torch.compile it is
    # evaluated while tracing and the graph keeps the answer
    return bool(nat.lib().tw_jeanie_fused_supported(K, T, U, D, fvm, features))


def _fused_saved_bytes(B, K, T, U, fvm, features):
    return int(nat.lib().tw_jeanie_fused_saved_bytes(B, K, T, U, int(fvm), int(features)))


@torch.library.custom_op("torchwarp_b200::jeanie_fused", mutates_args=())
def jeanie_fused(query: Optional[Tensor], support: Optional[Tensor], cost: Optional[Tensor],
                 K1: int, K2: int, T: int, U: int, s1: int, s2: int, gamma: float, metric: int,
                 fvm: bool, keep_R: bool) -> Tuple[Tensor, Tensor, Tensor]:
    """JEANIE (fvm False) or FVM (fvm True) on features (query [B, K1 K2 T, D],
    support [B, U, D]) or on a cost [B, K1, K2, T, U] ([B, K, T, U] for FVM).
    Returns (out [B], accumulator [B, K1, K2, T, U] or an empty tensor, saved
    state bytes)."""
    feat = query is not None
    ref = query if feat else cost
    nat.require_cuda(ref, support)
    B = ref.shape[0]
    D = query.shape[-1] if feat else 0
    q = query.contiguous() if feat else None
    s = support.contiguous() if feat else None
    c = None if feat else cost.contiguous()
    out = ref.new_empty(B)
    R = ref.new_empty(B, K1, K2, T, U) if (keep_R and not fvm) else ref.new_empty(0)
    sb = round_to_pairs(_fused_saved_bytes(B, K1 * K2, T, U, fvm, feat), B)
    saved = torch.empty(sb, dtype=torch.uint8, device=ref.device)
    if B:
        with torch.cuda.device(ref.device):
            nat.check(nat.call("jeanie_fused_forward", nat.lib().tw_jeanie_fused_forward_f32,
                               nat.ptr(q), nat.ptr(s), nat.ptr(c), B, K1, K2, T, U, D, s1, s2,
                               metric, int(fvm), float(gamma), nat.ptr(out),
                               nat.ptr(R) if R.numel() else None, nat.ptr(saved), sb,
                               nat.stream_of(ref)), "tw_jeanie_fused_forward")
    return out, R, saved


@jeanie_fused.register_fake
def _(query, support, cost, K1, K2, T, U, s1, s2, gamma, metric, fvm, keep_R):
    feat = query is not None
    ref = query if feat else cost
    B = ref.shape[0]
    sb = round_to_pairs(_fused_saved_bytes(B, K1 * K2, T, U, fvm, feat), B) if B else 0
    R = ref.new_empty(B, K1, K2, T, U) if (keep_R and not fvm) else ref.new_empty(0)
    return ref.new_empty(B), R, ref.new_empty(sb, dtype=torch.uint8)


@torch.library.custom_op("torchwarp_b200::jeanie_fused_backward", mutates_args=())
def jeanie_fused_backward(query: Optional[Tensor], support: Optional[Tensor],
                          cost: Optional[Tensor], saved: Tensor, grad_out: Tensor,
                          grad_R: Optional[Tensor], K1: int, K2: int, T: int, U: int, s1: int,
                          s2: int, gamma: float, metric: int,
                          fvm: bool) -> Tuple[Tensor, Tensor, Tensor]:
    """(d_query, d_support, d_cost) for L = sum grad_out * out + <grad_R, R>;
    the inputs that were not given come back as empty tensors."""
    feat = query is not None
    ref = query if feat else cost
    nat.require_cuda(ref, grad_out)
    B = ref.shape[0]
    D = query.shape[-1] if feat else 0
    q = query.contiguous() if feat else None
    s = support.contiguous() if feat else None
    c = None if feat else cost.contiguous()
    dq = torch.empty_like(q) if feat else ref.new_empty(0)
    ds = torch.empty_like(s) if feat else ref.new_empty(0)
    dC = ref.new_empty(0) if feat else torch.empty_like(c)
    if B:
        g_out = grad_out.to(ref.dtype).contiguous()
        gR = None if grad_R is None else grad_R.to(ref.dtype).contiguous()
        with torch.cuda.device(ref.device):
            nat.check(nat.call("jeanie_fused_backward", nat.lib().tw_jeanie_fused_backward_f32,
                               nat.ptr(q), nat.ptr(s), nat.ptr(c), nat.ptr(g_out), nat.ptr(gR), B,
                               K1, K2, T, U, D, s1, s2, metric, int(fvm), float(gamma),
                               nat.ptr(saved), saved.numel(), nat.ptr(dq) if feat else None,
                               nat.ptr(ds) if feat else None, None if feat else nat.ptr(dC),
                               nat.stream_of(ref)), "tw_jeanie_fused_backward")
    return dq, ds, dC


@jeanie_fused_backward.register_fake
def _(query, support, cost, saved, grad_out, grad_R, K1, K2, T, U, s1, s2, gamma, metric, fvm):
    feat = query is not None
    ref = query if feat else cost
    return ((torch.empty_like(query) if feat else ref.new_empty(0)),
            (torch.empty_like(support) if feat else ref.new_empty(0)),
            (ref.new_empty(0) if feat else torch.empty_like(cost)))


_register_autocast(jeanie_fused)
_register_autocast(jeanie_fused_backward)
register_fold_rule(jeanie_fused, flat_out=(2,), placeholder_out=(1,))
register_fold_rule(jeanie_fused_backward, flat_in=(3,), placeholder_out=(0, 1, 2))


class JeanieFused(torch.autograd.Function):
    """(query?, support?, cost?) -> (out, accumulator, saved): JEANIE or FVM in
    one native call per direction (float32).  The accumulator is
    differentiable when requested (keep_R).

    Forward mode: the tangent of the distance is the inner product of its
    gradient (one native backward with unit seeds) with the input tangents;
    with the accumulator requested, both tangents come from torch.func.jvp of
    the differentiable restatement.  Differentiating the backward again goes
    through the same restatement (native first-order values)."""

    generate_vmap_rule = True

    @staticmethod
    def forward(query, support, cost, K1, K2, T, U, s1, s2, gamma, metric, fvm, keep_R):
        return jeanie_fused(query, support, cost, K1, K2, T, U, s1, s2, gamma, metric, fvm,
                            keep_R)

    @staticmethod
    def setup_context(ctx, inputs, output):
        query, support, cost, K1, K2, T, U, s1, s2, gamma, metric, fvm, keep_R = inputs
        ctx.set_materialize_grads(False)
        ctx.mark_non_differentiable(output[2])
        if not keep_R or fvm:
            ctx.mark_non_differentiable(output[1])
        ctx.save_for_backward(query, support, cost, output[2])
        ctx.save_for_forward(query, support, cost, output[2])
        ctx.args = (K1, K2, T, U, s1, s2, gamma, metric, fvm, keep_R)

    @staticmethod
    def backward(ctx, g_out, g_R, _g_saved):
        query, support, cost, saved = ctx.saved_tensors
        K1, K2, T, U, s1, s2, gamma, metric, fvm, _ = ctx.args
        ref = query if query is not None else cost
        if g_out is None:
            g_out = ref.new_zeros(ref.shape[0])
        if torch.is_grad_enabled():
            grads = AD.first_order(_fused_grad_native(ctx.args), _fused_grad_ref(ctx.args), 1,
                                   saved, query, support, cost, g_out, g_R)
            if query is not None:
                return (grads[0], grads[1], None) + (None,) * 10
            return (None, None, grads[0]) + (None,) * 10
        return JeanieFused._backward_once(ctx, query, support, cost, saved, g_out, g_R)

    @staticmethod
    @_transforms.once_differentiable
    def _backward_once(ctx, query, support, cost, saved, g_out, g_R):
        K1, K2, T, U, s1, s2, gamma, metric, fvm, _ = ctx.args
        dq, ds, dC = jeanie_fused_backward(query, support, cost, saved, g_out, g_R, K1, K2, T, U,
                                           s1, s2, gamma, metric, fvm)
        if query is not None:
            return (dq, ds, None) + (None,) * 10
        return (None, None, dC) + (None,) * 10

    @staticmethod
    def jvp(ctx, q_t, s_t, c_t, *_):
        query, support, cost, saved = ctx.saved_tensors
        K1, K2, T, U, s1, s2, gamma, metric, fvm, keep_R = ctx.args
        if keep_R and not fvm:
            fwd = _fused_forward_ref(ctx.args, query is not None)
            if query is not None:
                prim = (query.contiguous(), support.contiguous())
                tans = (torch.zeros_like(query) if q_t is None else q_t.contiguous(),
                        torch.zeros_like(support) if s_t is None else s_t.contiguous())
            else:
                prim = (cost.contiguous(),)
                tans = (torch.zeros_like(cost) if c_t is None else c_t.contiguous(),)
            out_t, R_t = torch.func.jvp(fwd, prim, tans)[1]
            return out_t, R_t, None
        ref = query if query is not None else cost
        B = ref.shape[0]
        dq, ds, dC = jeanie_fused_backward(query, support, cost, saved, ref.new_ones(B), None, K1,
                                           K2, T, U, s1, s2, gamma, metric, fvm)
        t = ref.new_zeros(B)
        if query is not None:
            if q_t is not None:
                t = t + (dq * q_t).flatten(1).sum(1)
            if s_t is not None:
                t = t + (ds * s_t).flatten(1).sum(1)
        elif c_t is not None:
            t = t + (dC * c_t).flatten(1).sum(1)
        return t, None, None


def _fused_forward_ref(args, features):
    """Differentiable restatement of jeanie_fused's (out, R): a function of
    (query, support) with features, else of the cost."""
    K1, K2, T, U, s1, s2, gamma, metric, fvm, _ = args

    def from_cost(c):
        B = c.shape[0]
        if fvm:
            temporal = AD.viewpoint_softmin(c.reshape(B, K1 * K2, T, U), gamma)
            return AD.udtw_dp(temporal, None, gamma)[0], c.new_zeros(0)
        return AD.jeanie_dp(c.reshape(B, K1, K2, T, U), s1, s2, gamma)

    def from_features(q, s_):
        return from_cost(AD.qs_cost(q, s_, metric))

    return from_features if features else from_cost


def _fused_grad_native(args):
    """(saved, query, support, cost, g_out, g_R) -> the native gradients of
    the given inputs ((d_query, d_support) or (d_cost,))."""
    K1, K2, T, U, s1, s2, gamma, metric, fvm, _ = args

    def f(saved, q, s_, c, g_out, g_R):
        dq, ds, dC = jeanie_fused_backward(q, s_, c, saved, g_out, g_R, K1, K2, T, U, s1, s2,
                                           gamma, metric, fvm)
        return (dq, ds) if q is not None else (dC,)
    return f


def _fused_grad_ref(args):
    """The same gradients with differentiable torch operations."""
    K1, K2, T, U, s1, s2, gamma, metric, fvm, _ = args

    def f(saved, q, s_, c, g_out, g_R):
        def fwd_cost(cc):
            B = cc.shape[0]
            if fvm:
                temporal = AD.viewpoint_softmin(cc.reshape(B, K1 * K2, T, U), gamma)
                return (AD.udtw_dp(temporal, None, gamma)[0],)
            return AD.jeanie_dp(cc.reshape(B, K1, K2, T, U), s1, s2, gamma)

        cots = (g_out,) if fvm else (g_out, torch.zeros(
            (g_out.shape[0], K1, K2, T, U), dtype=g_out.dtype, device=g_out.device)
            if g_R is None else g_R)
        if q is not None:
            _, pull = torch.func.vjp(lambda a, b: fwd_cost(AD.qs_cost(a, b, metric)), q, s_)
        else:
            _, pull = torch.func.vjp(fwd_cost, c)
        return pull(cots)
    return f


JeanieFusedTraced = _transforms.traceable(JeanieFused)


def fused_apply(query, support, cost, K1, K2, T, U, s1, s2, gamma, metric, fvm, keep_R):
    """JeanieFused.apply (its traceable twin under torch.compile)."""
    return _transforms.pick(JeanieFused, JeanieFusedTraced).apply(
        query, support, cost, int(K1), int(K2), int(T), int(U), int(s1), int(s2), float(gamma),
        int(metric), bool(fvm), bool(keep_R))
