"""uDTW / soft-DTW as torch custom operators over the native C ABI.

Mirrors the reference op layer (hibana2077/torchwarp src/torchwarp/udtw/_ops.py:
custom ops ``dp``/``dp_backward``/``fused``/``fused_backward`` at :100-211,
autograd Functions at :262-415) with the native sm_100a kernels as the only
implementation:

* ``torchwarp_b200::sdtw_dp(cost, penalty?, gamma, bandwidth)`` ->
  (out_r [B], out_p [B], saved): the soft-min DP on a precomputed cost
  (and uDTW penalty).  ``saved`` is the kernel's opaque saved stream
  (uint8), replacing the reference's diagonal-major R and P.
* ``torchwarp_b200::sdtw_dp_backward(saved, grad_r, grad_p, N, M, gamma,
  has_penalty)`` -> (d_cost, d_penalty); d_penalty is an empty tensor when
  has_penalty is False (nothing is written for a penalty that does not exist).
* ``torchwarp_b200::udtw_fused(X, Y, vx?, vy?, gamma, beta, eps, bandwidth)``
  -> (out_r, out_p, saved, cost): cost built by the native cost kernel from
  the features, then the DP.  ``vx``/``vy`` None means unit variance and no
  penalty (soft-DTW).
* ``torchwarp_b200::udtw_fused_backward(...)`` -> (dX, dY, dvx, dvy).
* ``torchwarp_b200::sdtw_fused(X, Y, gamma, bandwidth)`` -> (out_r, saved,
  mask) and ``sdtw_fused_backward(X, Y, mask, saved, grad_r, gamma)`` ->
  (dX, dY): soft-DTW on features.  The backward keeps the cost's positivity
  mask (1 bit per cell) instead of the cost, which is freed after the DP
  forward.

Each op has a fake (meta) implementation for torch.compile, a vmap rule that
merges the vmapped dimension with the pairs (``torchwarp_b200._vmap``; the
saved stream's size is a multiple of the pair count so that it splits per
slice), and runs in float32 under autocast.  The autograd Functions let
torch.func generate their vmap rules from these.  First-order reverse mode
calls the native backward.

Higher-order derivatives of soft-DTW (no penalty), on a cost or on features,
are native too.  Differentiating through the backward (create_graph=True) is
a Hessian-vector product: with the incoming direction V as a uDTW penalty,
the penalty recursion ends at <E, V> (E = dd/dcost), and the native uDTW
backward of that value is H V.  Forward mode (jvp) is the same uDTW forward
with the tangent as the penalty, and for uDTW one native backward.  The
reference routes all of these through its pure-PyTorch autograd DP
(udtw/_ops.py:226-258, udtw/_autograd.py:32-79).  Second derivatives of uDTW
with a penalty, and third derivatives, raise.
"""

from typing import Optional, Tuple

import torch
from torch import Tensor

from .. import _native as nat
from .. import _autodiff as AD
from .. import _transforms
from .._vmap import register_fold_rule, round_to_pairs

# ------------------------------------------------------------------ helpers


def _saved_bytes(B, N, M, dtype, has_p):
    return int(nat.lib().tw_sdtw_saved_bytes(B, N, M, torch.empty((), dtype=dtype).element_size(),
                                             int(has_p)))


def _ws_bytes(B, N, M, dtype, has_p):
    return int(nat.lib().tw_sdtw_workspace_bytes(B, N, M,
                                                 torch.empty((), dtype=dtype).element_size(),
                                                 int(has_p)))


def _register_autocast(op):
    for device in ("cuda", "cpu"):
        torch.library.register_autocast(op, device, torch.float32)


def _dp_forward(cost, penalty, gamma, bandwidth):
    nat.require_cuda(cost, penalty)
    B, N, M = cost.shape
    cost = cost.contiguous()
    penalty = None if penalty is None else penalty.contiguous()
    has_p = penalty is not None
    out_r = cost.new_empty(B)
    out_p = cost.new_zeros(B)
    if B == 0:
        return out_r, out_p, torch.empty(0, dtype=torch.uint8, device=cost.device)
    with torch.cuda.device(cost.device):
        sb = round_to_pairs(_saved_bytes(B, N, M, cost.dtype, has_p), B)
        wb = _ws_bytes(B, N, M, cost.dtype, has_p)
        saved = torch.empty(sb, dtype=torch.uint8, device=cost.device)
        ws = torch.empty(wb, dtype=torch.uint8, device=cost.device)
        fn = getattr(nat.lib(), "tw_sdtw_forward_" + nat.suffix(cost.dtype))
        nat.check(nat.call("sdtw_forward", fn, nat.ptr(cost), nat.ptr(penalty), B, N, M,
                           float(gamma), float(bandwidth), nat.ptr(out_r),
                           nat.ptr(out_p) if has_p else None, nat.ptr(saved), sb, nat.ptr(ws), wb,
                           nat.stream_of(cost)), "tw_sdtw_forward")
    return out_r, out_p, saved


def _dp_backward(saved, grad_r, grad_p, N, M, gamma, has_p):
    """(d_cost [B,N,M], d_penalty): d_penalty is [B,N,M] with a penalty and an
    empty [0] tensor without one (soft-DTW has no penalty input to feed)."""
    nat.require_cuda(grad_r)
    B = grad_r.shape[0]
    dtype = grad_r.dtype
    d_cost = grad_r.new_empty(B, N, M)
    d_pen = grad_r.new_empty(B, N, M) if has_p else grad_r.new_empty(0)
    if B == 0:
        return d_cost, d_pen
    grad_r = grad_r.contiguous()
    grad_p = grad_p.to(dtype).contiguous()
    with torch.cuda.device(grad_r.device):
        wb = _ws_bytes(B, N, M, dtype, has_p)
        ws = torch.empty(wb, dtype=torch.uint8, device=grad_r.device)
        fn = getattr(nat.lib(), "tw_sdtw_backward_" + nat.suffix(dtype))
        nat.check(nat.call("sdtw_backward", fn, nat.ptr(grad_r),
                           nat.ptr(grad_p) if has_p else None, B, N, M, float(gamma), int(has_p),
                           nat.ptr(saved), saved.numel(), nat.ptr(d_cost),
                           nat.ptr(d_pen) if has_p else None, nat.ptr(ws), wb,
                           nat.stream_of(grad_r)), "tw_sdtw_backward")
    return d_cost, d_pen


def _dp_backward_flagged(saved, grad_r, grad_p, N, M, gamma, has_p):
    """fp32 _dp_backward through tw_sdtw_backward_flags_f32: also the chunk
    flags of d_cost / d_penalty for tw_udtw_features_grad_flagged_f32."""
    B = grad_r.shape[0]
    d_cost = grad_r.new_empty(B, N, M)
    d_pen = grad_r.new_empty(B, N, M) if has_p else grad_r.new_empty(0)
    grad_r = grad_r.contiguous()
    grad_p = grad_p.to(grad_r.dtype).contiguous()
    with torch.cuda.device(grad_r.device):
        lib = nat.lib()
        wb = _ws_bytes(B, N, M, grad_r.dtype, has_p)
        ws = torch.empty(wb, dtype=torch.uint8, device=grad_r.device)
        fb = lib.tw_sdtw_chunk_flags_bytes(B, N, M)
        flags = torch.empty(fb, dtype=torch.uint8, device=grad_r.device)
        nat.check(nat.call("sdtw_backward", lib.tw_sdtw_backward_flags_f32, nat.ptr(grad_r),
                           nat.ptr(grad_p) if has_p else None, B, N, M, float(gamma),
                           int(has_p), nat.ptr(saved), saved.numel(), nat.ptr(d_cost),
                           nat.ptr(d_pen) if has_p else None, nat.ptr(flags), fb, nat.ptr(ws),
                           wb, nat.stream_of(grad_r)), "tw_sdtw_backward_flags")
    return d_cost, d_pen, flags


# ------------------------------------------------- DP on precomputed matrices

@torch.library.custom_op("torchwarp_b200::sdtw_dp", mutates_args=())
def sdtw_dp(cost: Tensor, penalty: Optional[Tensor], gamma: float,
            bandwidth: float) -> Tuple[Tensor, Tensor, Tensor]:
    return _dp_forward(cost, penalty, gamma, bandwidth)


@sdtw_dp.register_fake
def _(cost, penalty, gamma, bandwidth):
    B, N, M = cost.shape
    nbytes = round_to_pairs(_saved_bytes(B, N, M, cost.dtype, penalty is not None), B) if B else 0
    return (cost.new_empty(B), cost.new_empty(B),
            cost.new_empty(nbytes, dtype=torch.uint8))


@torch.library.custom_op("torchwarp_b200::sdtw_dp_backward", mutates_args=())
def sdtw_dp_backward(saved: Tensor, grad_r: Tensor, grad_p: Tensor, N: int, M: int, gamma: float,
                     has_penalty: bool) -> Tuple[Tensor, Tensor]:
    return _dp_backward(saved, grad_r, grad_p, N, M, gamma, has_penalty)


@sdtw_dp_backward.register_fake
def _(saved, grad_r, grad_p, N, M, gamma, has_penalty):
    B = grad_r.shape[0]
    return grad_r.new_empty(B, N, M), (grad_r.new_empty(B, N, M) if has_penalty
                                       else grad_r.new_empty(0))


_register_autocast(sdtw_dp)
_register_autocast(sdtw_dp_backward)
register_fold_rule(sdtw_dp, flat_out=(2,))
register_fold_rule(sdtw_dp_backward, flat_in=(0,), placeholder_out=(1,))


# ------------------------------------- cost built from the features, then DP

@torch.library.custom_op("torchwarp_b200::udtw_fused", mutates_args=())
def udtw_fused(X: Tensor, Y: Tensor, vx: Optional[Tensor], vy: Optional[Tensor], gamma: float,
               beta: float, eps: float, bandwidth: float) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    nat.require_cuda(X, Y, vx, vy)
    B, N, D = X.shape
    M = Y.shape[1]
    X, Y = X.contiguous(), Y.contiguous()
    vx = None if vx is None else vx.contiguous()
    vy = None if vy is None else vy.contiguous()
    cost = X.new_empty(B, N, M)
    pen = X.new_empty(B, N, M) if vx is not None else None
    if B:
        with torch.cuda.device(X.device):
            fn = getattr(nat.lib(), "tw_udtw_cost_" + nat.suffix(X.dtype))
            nat.check(nat.call("udtw_cost", fn, nat.ptr(X), nat.ptr(Y), nat.ptr(vx), nat.ptr(vy),
                               B, N, M, D, float(beta), float(eps), nat.ptr(cost), nat.ptr(pen),
                               nat.stream_of(X)), "tw_udtw_cost")
    out_r, out_p, saved = _dp_forward(cost, pen, gamma, bandwidth)
    return out_r, out_p, saved, cost


@udtw_fused.register_fake
def _(X, Y, vx, vy, gamma, beta, eps, bandwidth):
    B, N, M = X.shape[0], X.shape[1], Y.shape[1]
    nbytes = round_to_pairs(_saved_bytes(B, N, M, X.dtype, vx is not None), B) if B else 0
    return (X.new_empty(B), X.new_empty(B), X.new_empty(nbytes, dtype=torch.uint8),
            X.new_empty(B, N, M))


@torch.library.custom_op("torchwarp_b200::udtw_fused_backward", mutates_args=())
def udtw_fused_backward(X: Tensor, Y: Tensor, vx: Optional[Tensor], vy: Optional[Tensor],
                        cost: Tensor, saved: Tensor, grad_r: Tensor, grad_p: Tensor, gamma: float,
                        beta: float, eps: float) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    B, N, D = X.shape
    M = Y.shape[1]
    has_p = vx is not None
    flags = None
    if X.dtype == torch.float32 and B:
        # fp32: the backward flags the chunks of dC / dQ holding a nonzero
        # value and the chain rule reads only those
        d_cost, d_pen, flags = _dp_backward_flagged(saved, grad_r, grad_p, N, M, gamma, has_p)
    else:
        d_cost, d_pen = _dp_backward(saved, grad_r, grad_p, N, M, gamma, has_p)
    X, Y = X.contiguous(), Y.contiguous()
    dX, dY = torch.empty_like(X), torch.empty_like(Y)
    dvx = torch.zeros_like(vx) if has_p else X.new_zeros(B, N)
    dvy = torch.zeros_like(vy) if has_p else X.new_zeros(B, M)
    if B:
        with torch.cuda.device(X.device):
            args = (nat.ptr(X), nat.ptr(Y), nat.ptr(vx.contiguous() if has_p else None),
                    nat.ptr(vy.contiguous() if has_p else None), nat.ptr(cost),
                    nat.ptr(d_cost), nat.ptr(d_pen) if has_p else None)
            tail = (B, N, M, D, float(beta), float(eps), nat.ptr(dX), nat.ptr(dY),
                    nat.ptr(dvx) if has_p else None, nat.ptr(dvy) if has_p else None,
                    nat.stream_of(X))
            if flags is not None:
                nat.check(nat.call("udtw_features_grad", nat.lib().tw_udtw_features_grad_flagged_f32,
                                   *args, nat.ptr(flags), *tail), "tw_udtw_features_grad_flagged")
            else:
                fn = getattr(nat.lib(), "tw_udtw_features_grad_" + nat.suffix(X.dtype))
                nat.check(nat.call("udtw_features_grad", fn, *args, *tail),
                          "tw_udtw_features_grad")
    return dX, dY, dvx, dvy


@udtw_fused_backward.register_fake
def _(X, Y, vx, vy, cost, saved, grad_r, grad_p, gamma, beta, eps):
    B, N, M = X.shape[0], X.shape[1], Y.shape[1]
    return (torch.empty_like(X), torch.empty_like(Y), X.new_empty(B, N), X.new_empty(B, M))


_register_autocast(udtw_fused)
_register_autocast(udtw_fused_backward)
register_fold_rule(udtw_fused, flat_out=(2,))
register_fold_rule(udtw_fused_backward, flat_in=(5,))


# ----------- soft-DTW from features: positivity mask instead of the saved cost

def _mask_words(M):
    return (M + 31) // 32


def _mask_rows(N):
    return (N + 3) // 4 * 4


@torch.library.custom_op("torchwarp_b200::sdtw_fused", mutates_args=())
def sdtw_fused(X: Tensor, Y: Tensor, gamma: float, bandwidth: float) -> Tuple[Tensor, Tensor,
                                                                              Tensor]:
    """soft-DTW on features: squared-Euclidean cost (tw_sqeuclid_cost) and the
    DP forward.  Returns (out_r [B], saved, mask [B, ceil(M/32), N] int32).
    The cost itself is dropped when the op returns: the backward needs only
    the saved stream and the cost's positivity mask."""
    nat.require_cuda(X, Y)
    B, N, D = X.shape
    M = Y.shape[1]
    X, Y = X.contiguous(), Y.contiguous()
    cost = X.new_empty(B, N, M)
    mask = torch.empty(B, _mask_words(M), _mask_rows(N), dtype=torch.int32, device=X.device)
    if B:
        with torch.cuda.device(X.device):
            fn = getattr(nat.lib(), "tw_sqeuclid_cost_" + nat.suffix(X.dtype))
            nat.check(nat.call("udtw_cost", fn, nat.ptr(X), nat.ptr(Y), B, N, M, D,
                               nat.ptr(cost), nat.ptr(mask), nat.stream_of(X)),
                      "tw_sqeuclid_cost")
    out_r, _, saved = _dp_forward(cost, None, gamma, bandwidth)
    return out_r, saved, mask


@sdtw_fused.register_fake
def _(X, Y, gamma, bandwidth):
    B, N, M = X.shape[0], X.shape[1], Y.shape[1]
    nbytes = round_to_pairs(_saved_bytes(B, N, M, X.dtype, False), B) if B else 0
    return (X.new_empty(B), X.new_empty(nbytes, dtype=torch.uint8),
            X.new_empty(B, _mask_words(M), _mask_rows(N), dtype=torch.int32))


@torch.library.custom_op("torchwarp_b200::sdtw_fused_backward", mutates_args=())
def sdtw_fused_backward(X: Tensor, Y: Tensor, mask: Tensor, saved: Tensor, grad_r: Tensor,
                        gamma: float) -> Tuple[Tensor, Tensor]:
    """(dX, dY).  The DP backward writes dL/dcost with the cost's positivity
    mask applied (tw_sdtw_backward_masked), so the chain rule takes it as S
    directly.  For fp32 the backward writes it sparsely, only the 8-column
    tiles that hold a nonzero value, with a bit mask of those values and
    flags of the chunks that hold them, and the chain rule reads only the
    flagged chunks and only the masked cells (tw_sdtw_backward_sparse_f32,
    tw_sqeuclid_grad_sparse_f32); the composition is
    tw_sdtw_features_backward."""
    nat.require_cuda(X, Y, grad_r)
    B, N, D = X.shape
    M = Y.shape[1]
    X, Y = X.contiguous(), Y.contiguous()
    dX, dY = torch.empty_like(X), torch.empty_like(Y)
    if B:
        dtype = X.dtype
        grad_r = grad_r.to(dtype).contiguous()
        s_cost = X.new_empty(B, N, M)
        with torch.cuda.device(X.device):
            lib = nat.lib()
            wb = _ws_bytes(B, N, M, dtype, False)
            ws = torch.empty(wb, dtype=torch.uint8, device=X.device)
            if dtype == torch.float32:
                fb = lib.tw_sdtw_chunk_flags_bytes(B, N, M)
                flags = torch.empty(fb, dtype=torch.uint8, device=X.device)
                nzm = torch.empty_like(mask)
                nat.check(nat.call("sdtw_backward", lib.tw_sdtw_backward_sparse_f32,
                                   nat.ptr(grad_r), B, N, M, float(gamma), nat.ptr(saved),
                                   saved.numel(), nat.ptr(mask), nat.ptr(s_cost), nat.ptr(nzm),
                                   nat.ptr(flags), fb, nat.ptr(ws), wb, nat.stream_of(X)),
                          "tw_sdtw_backward_sparse")
                nat.check(nat.call("udtw_features_grad", lib.tw_sqeuclid_grad_sparse_f32,
                                   nat.ptr(X), nat.ptr(Y), nat.ptr(nzm), nat.ptr(s_cost),
                                   nat.ptr(flags), B, N, M, D, nat.ptr(dX), nat.ptr(dY),
                                   nat.stream_of(X)),
                          "tw_sqeuclid_grad_sparse")
            else:
                fn = getattr(lib, "tw_sdtw_backward_masked_" + nat.suffix(dtype))
                nat.check(nat.call("sdtw_backward", fn, nat.ptr(grad_r), B, N, M, float(gamma),
                                   nat.ptr(saved), saved.numel(), nat.ptr(mask),
                                   nat.ptr(s_cost), nat.ptr(ws), wb, nat.stream_of(X)),
                          "tw_sdtw_backward_masked")
                fn = getattr(lib, "tw_sqeuclid_grad_" + nat.suffix(dtype))
                nat.check(nat.call("udtw_features_grad", fn, nat.ptr(X), nat.ptr(Y), None,
                                   nat.ptr(s_cost), B, N, M, D, nat.ptr(dX), nat.ptr(dY),
                                   nat.stream_of(X)), "tw_sqeuclid_grad")
    return dX, dY


@sdtw_fused_backward.register_fake
def _(X, Y, mask, saved, grad_r, gamma):
    return torch.empty_like(X), torch.empty_like(Y)


_register_autocast(sdtw_fused)
_register_autocast(sdtw_fused_backward)
register_fold_rule(sdtw_fused, flat_out=(1,))
register_fold_rule(sdtw_fused_backward, flat_in=(3,))


# ------------------------------------------------------- autograd Functions

def _zeros_if_none(g, like, B):
    return like.new_zeros(B) if g is None else g


def _pairwise_dot(a, b):
    """[B] sums of a * b over each pair's cells."""
    return (a * b).flatten(1).sum(1)


class SdtwCostGrad(torch.autograd.Function):
    """(cost, saved, g) -> g * dd/dcost for soft-DTW on a cost, differentiable
    once more with the native kernels.

    The backward is a Hessian-vector product.  Taking the direction V (the
    gradient that arrives for d_cost) as a uDTW penalty, the penalty recursion
    P_s = V_s + sum_p w_p P_p ends at <E, V> with E = dd/dcost.  The native
    uDTW forward returns that value, which is the gradient for g.  The native
    uDTW backward seeded with (0, g) returns g * (d^2 d / dcost^2) V, which is
    the gradient for the cost.  Third and higher derivatives, and forward
    mode through this backward (torch.func.hessian = jacfwd(jacrev)), go
    through torch.func on the differentiable restatement of the DP."""

    generate_vmap_rule = True

    @staticmethod
    def forward(cost, saved, g, gamma, bandwidth):
        B, N, M = cost.shape
        return sdtw_dp_backward(saved, g, g, N, M, gamma, False)[0]

    @staticmethod
    def setup_context(ctx, inputs, output):
        cost, saved, g, gamma, bandwidth = inputs
        ctx.save_for_backward(cost, g)
        ctx.save_for_forward(cost, g)
        ctx.args = (gamma, bandwidth)

    @staticmethod
    def _ref(gamma, bandwidth):
        """(cost, g) -> g * dd/dcost with differentiable torch operations."""
        def f(cost, g):
            _, pull = torch.func.vjp(lambda c: AD.udtw_dp(c, None, gamma, bandwidth)[0], cost)
            return pull(g)[0]
        return f

    @staticmethod
    def backward(ctx, V):
        cost, g = ctx.saved_tensors
        gamma, bandwidth = ctx.args
        if torch.is_grad_enabled():
            # a third derivative follows: the same products, differentiable
            _, pull = torch.func.vjp(SdtwCostGrad._ref(gamma, bandwidth), cost, g)
            hv, v_e = pull(V.to(cost.dtype))
            return hv, None, v_e, None, None
        return SdtwCostGrad._native_hvp(cost, g, V, gamma, bandwidth)

    @staticmethod
    def _native_hvp(cost, g, V, gamma, bandwidth):
        B, N, M = cost.shape
        _, v_e, saved_v = sdtw_dp(cost, V.to(cost.dtype), gamma, bandwidth)
        hv, _ = sdtw_dp_backward(saved_v, torch.zeros_like(g), g, N, M, gamma, True)
        return hv, None, v_e, None, None

    @staticmethod
    def jvp(ctx, cost_t, _saved_t, g_t, _gamma_t, _bandwidth_t):
        cost, g = ctx.saved_tensors
        gamma, bandwidth = ctx.args
        cost_t = torch.zeros_like(cost) if cost_t is None else cost_t.to(cost.dtype)
        g_t = torch.zeros_like(g) if g_t is None else g_t.to(g.dtype)
        return torch.func.jvp(SdtwCostGrad._ref(gamma, bandwidth),
                              (cost.contiguous(), g.contiguous()),
                              (cost_t.contiguous(), g_t.contiguous()))[1]


def _dp_grad_native(N, M, gamma):
    """(saved, cost, penalty, g_r, g_p) -> (d_cost, d_penalty), native."""
    def f(saved, cost, penalty, g_r, g_p):
        return sdtw_dp_backward(saved, g_r, g_p, N, M, gamma, True)
    return f


def _dp_grad_ref(gamma, bandwidth):
    """(saved, cost, penalty, g_r, g_p) -> (d_cost, d_penalty), differentiable."""
    def f(saved, cost, penalty, g_r, g_p):
        _, pull = torch.func.vjp(lambda c, q: AD.udtw_dp(c, q, gamma, bandwidth), cost, penalty)
        return pull((g_r, g_p))
    return f


@_transforms.once_differentiable
def _dp_backward_once(ctx, saved, g_r, g_p):
    gamma, has_p, _ = ctx.args
    B, N, M = ctx.shape
    like = saved.new_empty(0, dtype=ctx.dtype)
    g_r = _zeros_if_none(g_r, like, B).to(ctx.dtype)
    g_p = _zeros_if_none(g_p, like, B).to(ctx.dtype)
    d_cost, d_pen = sdtw_dp_backward(saved, g_r, g_p, N, M, gamma, has_p)
    return d_cost, (d_pen if has_p else None), None, None


class DP(torch.autograd.Function):
    """(cost, penalty?) -> (distance, penalty_sum, saved)."""

    generate_vmap_rule = True

    @staticmethod
    def forward(cost, penalty, gamma, bandwidth):
        return sdtw_dp(cost, penalty, gamma, bandwidth)

    @staticmethod
    def setup_context(ctx, inputs, output):
        cost, penalty, gamma, bandwidth = inputs
        ctx.mark_non_differentiable(output[2])
        ctx.set_materialize_grads(False)
        # the cost is kept for a backward that is differentiated again (soft-DTW)
        ctx.save_for_backward(output[2], cost, penalty)
        if penalty is None:
            ctx.save_for_forward(cost, output[2])
        else:
            ctx.save_for_forward(cost, penalty, output[2])
        ctx.shape = tuple(cost.shape)
        ctx.dtype = cost.dtype
        ctx.args = (gamma, penalty is not None, bandwidth)

    @staticmethod
    def backward(ctx, g_r, g_p, _g_saved):
        saved, cost, penalty = ctx.saved_tensors
        gamma, has_p, bandwidth = ctx.args
        if torch.is_grad_enabled() and not has_p:
            # create_graph: a backward that is itself differentiable (natively)
            g = _zeros_if_none(g_r, cost, ctx.shape[0]).to(ctx.dtype)
            return SdtwCostGrad.apply(cost, saved, g, gamma, bandwidth), None, None, None
        if torch.is_grad_enabled():
            # uDTW: native values, higher orders through the restatement
            B, N, M = ctx.shape
            g_r = _zeros_if_none(g_r, cost, B).to(ctx.dtype)
            g_p = _zeros_if_none(g_p, cost, B).to(ctx.dtype)
            d_cost, d_pen = AD.first_order(_dp_grad_native(N, M, gamma),
                                           _dp_grad_ref(gamma, bandwidth), 1, saved, cost,
                                           penalty, g_r, g_p)
            return d_cost, d_pen, None, None
        return _dp_backward_once(ctx, saved, g_r, g_p)

    @staticmethod
    def jvp(ctx, cost_t, penalty_t, _gamma_t, _bandwidth_t):
        gamma, has_p, bandwidth = ctx.args
        B, N, M = ctx.shape
        if not has_p:
            cost, _ = ctx.saved_tensors
            # the penalty-sum output is a differentiable zero without a
            # penalty; it gets a zero tangent (None there trips forward mode)
            if cost_t is None:
                return cost.new_zeros(B), cost.new_zeros(B), None
            # d/de d(cost + e T) = <E, T>: the uDTW forward with T as the penalty
            _, r_t, _ = sdtw_dp(cost, cost_t.to(cost.dtype), gamma, bandwidth)
            return r_t, torch.zeros_like(r_t), None
        cost, penalty, saved = ctx.saved_tensors
        # one native backward of the penalty sum: dp/dcost, and dp/dpenalty = E
        d_cost, e = sdtw_dp_backward(saved, cost.new_zeros(B), cost.new_ones(B), N, M, gamma,
                                     True)
        r_t = cost.new_zeros(B)
        p_t = cost.new_zeros(B)
        if cost_t is not None:
            r_t = r_t + _pairwise_dot(e, cost_t)
            p_t = p_t + _pairwise_dot(d_cost, cost_t)
        if penalty_t is not None:
            p_t = p_t + _pairwise_dot(e, penalty_t)
        return r_t, p_t, None


class Fused(torch.autograd.Function):
    """(X, Y, vx?, vy?) -> (distance, penalty_sum, saved, cost).

    Differentiating the backward again (create_graph) rebuilds the cost and
    penalty as differentiable expressions and routes the DP part through
    the native backward with higher orders through the restatement; forward
    mode forms the cost's tangent and contracts it with the native
    gradients of both outputs."""

    generate_vmap_rule = True

    @staticmethod
    def forward(X, Y, vx, vy, gamma, beta, eps, bandwidth):
        return udtw_fused(X, Y, vx, vy, gamma, beta, eps, bandwidth)

    @staticmethod
    def setup_context(ctx, inputs, output):
        X, Y, vx, vy, gamma, beta, eps, bandwidth = inputs
        ctx.mark_non_differentiable(output[2], output[3])
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(X, Y, vx, vy, output[2], output[3])
        ctx.save_for_forward(X, Y, vx, vy, output[2])
        ctx.args = (gamma, beta, eps, bandwidth)

    @staticmethod
    def backward(ctx, g_r, g_p, _g_saved, _g_cost):
        X, Y, vx, vy, saved, cost = ctx.saved_tensors
        if torch.is_grad_enabled() and vx is not None:
            return Fused._backward_graph(ctx, X, Y, vx, vy, saved, g_r, g_p)
        return Fused._backward_once(ctx, X, Y, vx, vy, saved, cost, g_r, g_p)

    @staticmethod
    def _backward_graph(ctx, X, Y, vx, vy, saved, g_r, g_p):
        """Gradients that can be differentiated again (reverse or forward
        mode): the cost and penalty rebuilt with torch operations, the DP
        part native with higher orders through the restatement, and the
        chain rule by torch.func.vjp (each argument slot its own partial
        derivative, so normalize's d(X, X) is right)."""
        gamma, beta, eps, bandwidth = ctx.args
        B, N, M = X.shape[0], X.shape[1], Y.shape[1]
        g_r = _zeros_if_none(g_r, X, B).to(X.dtype)
        g_p = _zeros_if_none(g_p, X, B).to(X.dtype)

        def mats(a, b, c, d):
            with _full_fp32_matmul():
                return AD.udtw_matrices(a, b, c, d, beta, eps)

        (cost, pen), pull = torch.func.vjp(mats, X, Y, vx, vy)
        d_cost, d_pen = AD.first_order(_dp_grad_native(N, M, gamma),
                                       _dp_grad_ref(gamma, bandwidth), 1, saved, cost, pen,
                                       g_r, g_p)
        with _full_fp32_matmul():
            dX, dY, dvx, dvy = pull((d_cost, d_pen))
        return dX, dY, dvx, dvy, None, None, None, None

    @staticmethod
    def jvp(ctx, X_t, Y_t, vx_t, vy_t, *_):
        X, Y, vx, vy, saved = ctx.saved_tensors
        gamma, beta, eps, bandwidth = ctx.args
        B, N, M = X.shape[0], X.shape[1], Y.shape[1]
        prim = [t for t in (X, Y, vx, vy) if t is not None]
        tans = [torch.zeros_like(p) if t is None else t.to(p.dtype)
                for p, t in zip(prim, [X_t, Y_t, vx_t, vy_t])]
        if vx is None:
            cost_t = torch.func.jvp(AD.sq_euclid, tuple(p.contiguous() for p in prim),
                                    tuple(t.contiguous() for t in tans))[1]
            d_cost, _ = sdtw_dp_backward(saved, X.new_ones(B), X.new_zeros(B), N, M, gamma,
                                         False)
            return _pairwise_dot(d_cost, cost_t), X.new_zeros(B), None, None
        (cost_t, pen_t) = torch.func.jvp(
            lambda a, b, c, d: AD.udtw_matrices(a, b, c, d, beta, eps),
            tuple(p.contiguous() for p in prim), tuple(t.contiguous() for t in tans))[1]
        # gradients of both outputs: E = dd/dcost = dp/dpenalty, and dp/dcost
        e, _ = sdtw_dp_backward(saved, X.new_ones(B), X.new_zeros(B), N, M, gamma, True)
        dp_dc, _ = sdtw_dp_backward(saved, X.new_zeros(B), X.new_ones(B), N, M, gamma, True)
        return (_pairwise_dot(e, cost_t), _pairwise_dot(dp_dc, cost_t) + _pairwise_dot(e, pen_t),
                None, None)

    @staticmethod
    @_transforms.once_differentiable
    def _backward_once(ctx, X, Y, vx, vy, saved, cost, g_r, g_p):
        gamma, beta, eps, bandwidth = ctx.args
        B = X.shape[0]
        if cost is None:
            cost = ctx.saved_tensors[5]
        g_r = _zeros_if_none(g_r, X, B)
        g_p = _zeros_if_none(g_p, X, B)
        dX, dY, dvx, dvy = udtw_fused_backward(X, Y, vx, vy, cost, saved, g_r, g_p, gamma, beta,
                                               eps)
        has_p = vx is not None
        return dX, dY, (dvx if has_p else None), (dvy if has_p else None), None, None, None, None


class _full_fp32_matmul:
    """Context in which float32 matmuls run in full float32 (no TF32), so the
    cost rebuilt for a differentiable backward agrees with the native cost
    kernel (3xTF32, float32 accuracy) whatever the caller's TF32 setting."""

    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev


def _sqeuclid(X, Y):
    """||x_i - y_j||^2 clamped at 0, the native cost's formula, as a
    differentiable expression (its GEMM runs in cuBLAS, in full float32)."""
    x2 = (X * X).sum(-1)
    y2 = (Y * Y).sum(-1)
    with _full_fp32_matmul():
        G = torch.bmm(X, Y.transpose(1, 2))
    return (x2[:, :, None] + y2[:, None, :] - 2.0 * G).clamp_min(0)


@_transforms.once_differentiable
def _sdtw_fused_backward_once(ctx, X, Y, mask, saved, g_r):
    g_r = _zeros_if_none(g_r, X, X.shape[0])
    dX, dY = sdtw_fused_backward(X, Y, mask, saved, g_r, ctx.gamma)
    return dX, dY, None, None


class SdtwFused(torch.autograd.Function):
    """(X, Y) -> (distance, saved, mask): soft-DTW with squared-Euclidean cost."""

    generate_vmap_rule = True

    @staticmethod
    def forward(X, Y, gamma, bandwidth):
        return sdtw_fused(X, Y, gamma, bandwidth)

    @staticmethod
    def setup_context(ctx, inputs, output):
        X, Y, gamma, bandwidth = inputs
        ctx.mark_non_differentiable(output[1], output[2])
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(X, Y, output[2], output[1])
        ctx.save_for_forward(X, Y)
        ctx.gamma = gamma
        ctx.bandwidth = bandwidth

    @staticmethod
    def backward(ctx, g_r, _g_saved, _g_mask):
        X, Y, mask, saved = ctx.saved_tensors
        if not torch.is_grad_enabled():
            return _sdtw_fused_backward_once(ctx, X, Y, mask, saved, g_r)
        # create_graph (or torch.func): the cost is rebuilt as a differentiable
        # expression and the DP part goes through SdtwCostGrad, whose own
        # backward is native; torch.func.vjp applies the cost's chain rule,
        # each argument slot getting its own partial derivative (with X
        # passed as both arguments, normalize=True's d(X, X))
        g = _zeros_if_none(g_r, X, X.shape[0]).to(X.dtype)
        cost, pull = torch.func.vjp(_sqeuclid, X, Y)
        s = SdtwCostGrad.apply(cost, saved, g, ctx.gamma, ctx.bandwidth)
        with _full_fp32_matmul():
            dX, dY = pull(s)
        return dX, dY, None, None

    @staticmethod
    def jvp(ctx, X_t, Y_t, _gamma_t, _bandwidth_t):
        X, Y = ctx.saved_tensors
        B = X.shape[0]
        if X_t is None and Y_t is None:
            return X.new_zeros(B), None, None
        X_t = torch.zeros_like(X) if X_t is None else X_t.to(X.dtype)
        Y_t = torch.zeros_like(Y) if Y_t is None else Y_t.to(Y.dtype)
        cost = _sqeuclid(X, Y)
        # the cost's tangent, zero where the clamp holds it at 0
        cost_t = (2.0 * (X * X_t).sum(-1)[:, :, None] + 2.0 * (Y * Y_t).sum(-1)[:, None, :]
                  - 2.0 * (torch.bmm(X_t, Y.transpose(1, 2)) + torch.bmm(X, Y_t.transpose(1, 2))))
        cost_t = torch.where(cost > 0, cost_t, torch.zeros_like(cost_t))
        _, r_t, _ = sdtw_dp(cost, cost_t, ctx.gamma, ctx.bandwidth)
        return r_t, None, None


DPTraced = _transforms.traceable(DP)
FusedTraced = _transforms.traceable(Fused)
SdtwFusedTraced = _transforms.traceable(SdtwFused)


def sdtw_fused_apply(X, Y, gamma, bandwidth):
    return _transforms.pick(SdtwFused, SdtwFusedTraced).apply(X, Y, gamma, bandwidth)


def dp_apply(cost, penalty, gamma, bandwidth):
    return _transforms.pick(DP, DPTraced).apply(cost, penalty, gamma, bandwidth)


def fused_apply(X, Y, vx, vy, gamma, beta, eps, bandwidth):
    return _transforms.pick(Fused, FusedTraced).apply(X, Y, vx, vy, gamma, beta, eps, bandwidth)
