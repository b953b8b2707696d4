"""vmap rules of the custom operators (torchwarp_b200._vmap), on the CPU.

The native operators need a GPU, so the rules are exercised here on a toy
pair of operators with the same structure: a forward that returns a value
per pair and an opaque byte buffer laid out across pairs (here, the inputs
transposed, so that no slice of it belongs to one pair), and a backward that
reads that buffer.  The tests cover a vmapped forward, per-sample gradients
(vmap of grad), vmapped cotangents of an unbatched forward (jacrev: one
backward per slice), nested vmaps and the buffer-size rounding.
"""

import pytest
import torch
from torch import Tensor

from torchwarp_b200._vmap import register_fold_rule, round_to_pairs

f64 = torch.float64


@torch.library.custom_op("twtest::pair_fwd", mutates_args=())
def pair_fwd(x: Tensor) -> tuple[Tensor, Tensor]:
    """(x [B, n]) -> (sum of squares [B], saved bytes: x^T, padded)."""
    B, n = x.shape
    raw = x.t().contiguous().view(torch.uint8).reshape(-1)
    saved = torch.zeros(round_to_pairs(raw.numel(), B), dtype=torch.uint8)
    saved[:raw.numel()] = raw
    return (x * x).sum(1), saved


@pair_fwd.register_fake
def _(x):
    B, n = x.shape
    return x.new_empty(B), x.new_empty(round_to_pairs(B * n * 8, B), dtype=torch.uint8)


@torch.library.custom_op("twtest::pair_bwd", mutates_args=())
def pair_bwd(saved: Tensor, g: Tensor, n: int) -> tuple[Tensor, Tensor]:
    """(saved, g [B], n) -> (dx [B, n] = 2 x g, empty placeholder)."""
    B = g.shape[0]
    x = saved[:B * n * 8].view(f64).reshape(n, B).t()
    return 2.0 * x * g[:, None], g.new_empty(0)


@pair_bwd.register_fake
def _(saved, g, n):
    return g.new_empty(g.shape[0], n), g.new_empty(0)


register_fold_rule(pair_fwd, flat_out=(1,))
register_fold_rule(pair_bwd, flat_in=(0,), placeholder_out=(1,))


class PairSq(torch.autograd.Function):
    generate_vmap_rule = True

    @staticmethod
    def forward(x):
        return pair_fwd(x)

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.mark_non_differentiable(output[1])
        ctx.save_for_backward(output[1])
        ctx.n = inputs[0].shape[1]

    @staticmethod
    def backward(ctx, g, _g_saved):
        (saved,) = ctx.saved_tensors
        return pair_bwd(saved, g, ctx.n)[0]


def f(x):
    return PairSq.apply(x)[0]


@torch.library.custom_op("twtest::pair_dist", mutates_args=())
def pair_dist(q: Tensor, s: Tensor) -> Tensor:
    """A single-result op: (q [B, R, D], s [B, U, D]) -> [B, R, U]."""
    return torch.cdist(q, s)


@pair_dist.register_fake
def _(q, s):
    return q.new_empty(q.shape[0], q.shape[1], s.shape[1])


register_fold_rule(pair_dist)


class PairDist(torch.autograd.Function):
    generate_vmap_rule = True

    @staticmethod
    def forward(q, s):
        return pair_dist(q, s)

    @staticmethod
    def setup_context(ctx, inputs, output):
        pass

    @staticmethod
    def backward(ctx, g):
        return None, None


def test_round_to_pairs():
    assert round_to_pairs(0, 5) == 0
    assert round_to_pairs(10, 5) == 10
    assert round_to_pairs(11, 5) == 15
    assert round_to_pairs(7, 1) == 7 and round_to_pairs(7, 0) == 7


def test_vmapped_forward():
    x = torch.randn(3, 4, 5, dtype=f64)
    got = torch.func.vmap(f)(x)
    assert torch.equal(got, (x * x).sum(-1))


def test_vmapped_forward_saved_splits_per_slice():
    # 3 slices of 5 pairs of 7 values: 3 * 5 * 7 * 8 = 840 bytes over 15 pairs
    x = torch.randn(3, 5, 7, dtype=f64)
    _, saved = torch.func.vmap(pair_fwd)(x)
    assert saved.shape == (3, 280)


def test_per_sample_grad():
    x = torch.randn(4, 2, 6, dtype=f64)
    g = torch.func.vmap(torch.func.grad(lambda a: f(a).sum()))(x)
    assert torch.allclose(g, 2.0 * x)


def test_jacrev_loops_over_cotangents():
    # unbatched forward, vmapped cotangents: the backward sees the saved
    # buffer unbatched and runs once per slice
    x = torch.randn(3, 4, dtype=f64)
    J = torch.func.jacrev(f)(x)
    want = torch.zeros(3, 3, 4, dtype=f64)
    for b in range(3):
        want[b, b] = 2.0 * x[b]
    assert torch.allclose(J, want)


def test_nested_vmap():
    x = torch.randn(2, 3, 5, 4, dtype=f64)
    got = torch.func.vmap(torch.func.vmap(f))(x)
    assert torch.equal(got, (x * x).sum(-1))
    g = torch.func.vmap(torch.func.vmap(torch.func.grad(lambda a: f(a).sum())))(x)
    assert torch.allclose(g, 2.0 * x)


def test_unbatched_pair_argument_is_expanded():
    saved_x = torch.randn(3, 4, dtype=f64)
    _, saved = pair_fwd(saved_x)
    gs = torch.randn(2, 3, dtype=f64)   # vmapped cotangents; saved unbatched -> loop
    dx, ph = torch.func.vmap(pair_bwd, in_dims=(None, 0, None))(saved, gs, 4)
    assert torch.allclose(dx, 2.0 * saved_x[None] * gs[:, :, None])
    assert ph.shape == (2, 0)


@pytest.mark.parametrize("V", [1, 2, 3, 7])
def test_any_slice_count(V):
    x = torch.randn(V, 3, 5, dtype=f64)
    g = torch.func.vmap(torch.func.grad(lambda a: f(a).sum()))(x)
    assert torch.allclose(g, 2.0 * x)


def test_single_result_op_through_reshapes():
    # the query/support layout of JEANIE: views and expands before the op
    q = torch.randn(3, 2, 4, 5, 3, dtype=f64)
    s = torch.randn(3, 2, 6, 3, dtype=f64)

    def cost(a, b):
        B, K, T, D = a.shape
        sp = b.unsqueeze(-3).expand(B, 1, 6, D).reshape(-1, 6, D)
        return PairDist.apply(a.reshape(B, K * T, D), sp).reshape(B, K, T, 6)

    got = torch.func.vmap(cost)(q, s)
    want = torch.cdist(q.reshape(3, 2, 20, 3), s).reshape(3, 2, 4, 5, 6)
    assert torch.allclose(got, want)


# ---------------------------------------------- first-order-only backwards

from torchwarp_b200 import _transforms  # noqa: E402


class OnceSq(torch.autograd.Function):
    generate_vmap_rule = True

    @staticmethod
    def forward(x):
        return x * x

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.save_for_backward(inputs[0])

    @staticmethod
    @_transforms.once_differentiable
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return 2 * x * g


def test_once_differentiable_first_order_under_torch_func():
    x = torch.randn(3, 4, dtype=f64)
    f = lambda a: OnceSq.apply(a).sum()  # noqa: E731
    assert torch.allclose(torch.func.grad(f)(x), 2 * x)
    assert torch.allclose(torch.func.vmap(torch.func.grad(f))(x), 2 * x)
    J = torch.func.jacrev(OnceSq.apply)(x[0])
    assert torch.allclose(J, torch.diag(2 * x[0]))


def test_once_differentiable_second_order_raises():
    x = torch.randn(4, dtype=f64)
    f = lambda a: OnceSq.apply(a).sum()  # noqa: E731
    with pytest.raises(RuntimeError, match="differentiate twice"):
        torch.func.jacrev(torch.func.jacrev(f))(x)
    with pytest.raises(RuntimeError, match="differentiate twice"):
        torch.func.grad(lambda a: torch.func.grad(f)(a).sum())(x)
    y = x.clone().requires_grad_(True)
    (gy,) = torch.autograd.grad(f(y), y, create_graph=True)
    with pytest.raises(RuntimeError):
        gy.sum().backward()
