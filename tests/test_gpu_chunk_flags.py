"""Nonzero-chunk flags of dL/dcost and the chain rule that skips the chunks
flagged zero (fp32 soft-DTW on features, B200).

The DP backward flags every 128 x 32 (and 32 x 128) chunk of dL/dcost it
writes a nonzero value into; the tensor-core chain rule
(dX = -2 S Y + 2 X rowsum(S), dY = -2 S^T X + 2 Y colsum(S), the reference's
_features_grads, hibana2077/torchwarp src/torchwarp/udtw/_ops.py:179-183)
reads only those chunks and the first chunk of each unit.  A skipped chunk
holds only zeros, so the result must equal the dense product bit for bit.
"""

import numpy as np
import pytest
import torch

from torchwarp_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _round16(n):
    return (n + 15) // 16 * 16


def _align256(n):
    return (n + 255) // 256 * 256


def _flags_ref(S):
    """The flag bytes tw_sdtw_backward_masked_flags_f32 must write for S [B, N, M]."""
    B, N, M = S.shape
    nz = (S != 0).cpu().numpy()
    kr, kc = _round16(-(-M // 32)), _round16(-(-N // 32))
    nr, nc = -(-N // 128), -(-M // 128)
    rows = np.zeros((B, nr, kr), np.uint8)
    cols = np.zeros((B, nc, kc), np.uint8)
    for b in range(B):
        for i0 in range(0, N, 128):
            for j0 in range(0, M, 32):
                rows[b, i0 // 128, j0 // 32] = nz[b, i0:i0 + 128, j0:j0 + 32].any()
        for j0 in range(0, M, 128):
            for i0 in range(0, N, 32):
                cols[b, j0 // 128, i0 // 32] = nz[b, i0:i0 + 32, j0:j0 + 128].any()
    out = np.zeros(_align256(rows.size) + _align256(cols.size), np.uint8)
    out[:rows.size] = rows.ravel()
    out[_align256(rows.size):_align256(rows.size) + cols.size] = cols.ravel()
    return out


def _inputs(B, N, M, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(B, N, D, device="cuda", generator=g),
            torch.randn(B, M, D, device="cuda", generator=g))


def _forward(X, Y, gamma):
    lib = nat.lib()
    B, N, D = X.shape
    M = Y.shape[1]
    C = torch.empty(B, N, M, device="cuda")
    mask = torch.empty(B, -(-M // 32), (N + 3) // 4 * 4, dtype=torch.int32, device="cuda")
    nat.check(lib.tw_sqeuclid_cost_f32(nat.ptr(X), nat.ptr(Y), B, N, M, D, nat.ptr(C),
                                       nat.ptr(mask), nat.stream_of(X)), "tw_sqeuclid_cost_f32")
    sb = lib.tw_sdtw_saved_bytes(B, N, M, 4, 0)
    wb = lib.tw_sdtw_workspace_bytes(B, N, M, 4, 0)
    saved = torch.empty(sb, dtype=torch.uint8, device="cuda")
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    out = torch.empty(B, device="cuda")
    nat.check(lib.tw_sdtw_forward_f32(nat.ptr(C), None, B, N, M, float(gamma), 0.0, nat.ptr(out),
                                      None, nat.ptr(saved), sb, nat.ptr(ws), wb,
                                      nat.stream_of(X)), "tw_sdtw_forward_f32")
    return mask, saved, ws


def _backward(X, Y, gamma, flagged):
    lib = nat.lib()
    B, N, _ = X.shape
    M = Y.shape[1]
    mask, saved, ws = _forward(X, Y, gamma)
    g = torch.linspace(0.5, 1.5, B, device="cuda")
    dC = torch.empty(B, N, M, device="cuda")
    if not flagged:
        nat.check(lib.tw_sdtw_backward_masked_f32(nat.ptr(g), B, N, M, float(gamma),
                                                  nat.ptr(saved), saved.numel(), nat.ptr(mask),
                                                  nat.ptr(dC), nat.ptr(ws), ws.numel(),
                                                  nat.stream_of(X)), "backward_masked")
        return dC, None
    fb = lib.tw_sdtw_chunk_flags_bytes(B, N, M)
    flags = torch.full((fb,), 7, dtype=torch.uint8, device="cuda")  # zeroed by the call
    nat.check(lib.tw_sdtw_backward_masked_flags_f32(nat.ptr(g), B, N, M, float(gamma),
                                                    nat.ptr(saved), saved.numel(), nat.ptr(mask),
                                                    nat.ptr(dC), nat.ptr(flags), fb, nat.ptr(ws),
                                                    ws.numel(), nat.stream_of(X)),
              "backward_masked_flags")
    return dC, flags


def _grad(X, Y, dC, flags):
    B, N, D = X.shape
    M = Y.shape[1]
    dX, dY = torch.empty_like(X), torch.empty_like(Y)
    if flags is None:
        st = nat.lib().tw_sqeuclid_grad_f32(nat.ptr(X), nat.ptr(Y), None, nat.ptr(dC), B, N, M, D,
                                            nat.ptr(dX), nat.ptr(dY), nat.stream_of(X))
    else:
        st = nat.lib().tw_sqeuclid_grad_flagged_f32(nat.ptr(X), nat.ptr(Y), nat.ptr(dC),
                                                    nat.ptr(flags), B, N, M, D, nat.ptr(dX),
                                                    nat.ptr(dY), nat.stream_of(X))
    nat.check(st, "chain rule")
    torch.cuda.synchronize()
    return dX, dY


CASES = [  # B, N, M, D, gamma
    (3, 256, 256, 64, 0.01),    # near-hard alignment: most chunks zero
    (2, 200, 300, 64, 0.01),    # ragged rows and columns
    (2, 160, 192, 64, 1.0),     # soft alignment: every chunk nonzero
    (2, 130, 140, 128, 0.01),   # S in shared memory (wide MMAs)
    (1, 96, 260, 256, 0.01),    # S in shared memory, narrow MMAs
    (1, 1, 4, 64, 0.01),
]


@pytest.mark.parametrize("case", CASES)
def test_flags_mark_exactly_the_nonzero_chunks(case):
    B, N, M, D, gamma = case
    X, Y = _inputs(B, N, M, D, 11)
    dC0, _ = _backward(X, Y, gamma, flagged=False)
    dC, flags = _backward(X, Y, gamma, flagged=True)
    torch.cuda.synchronize()
    assert torch.equal(dC, dC0)
    np.testing.assert_array_equal(flags.cpu().numpy(), _flags_ref(dC))


@pytest.mark.parametrize("case", CASES)
def test_flagged_chain_rule_equals_dense(case, monkeypatch):
    B, N, M, D, gamma = case
    X, Y = _inputs(B, N, M, D, 12)
    dC, flags = _backward(X, Y, gamma, flagged=True)
    monkeypatch.delenv("TW_GRAD_DENSE", raising=False)
    got = _grad(X, Y, dC, flags)
    dense = _grad(X, Y, dC, None)
    monkeypatch.setenv("TW_GRAD_DENSE", "1")
    forced = _grad(X, Y, dC, flags)
    for a, b, c in zip(got, dense, forced):
        assert torch.equal(a, b)
        assert torch.equal(c, b)


@pytest.mark.parametrize("shape", [(1, 128, 4096, 64), (1, 4096, 128, 64), (2, 300, 2200, 64)])
def test_flag_windows_beyond_64_chunks(shape):
    """Hand-made sparse S whose nonzero chunks sit at window edges (chunk 0,
    63, 64, the last) on the long side, so the schedule crosses several
    64-chunk flag windows in both chain-rule directions."""
    B, N, M, D = shape
    X, Y = _inputs(B, N, M, D, 13)
    S = torch.zeros(B, N, M, device="cuda")
    g = torch.Generator().manual_seed(5)
    for b in range(B):
        for j in {0, 31, 32 * 63, 32 * 64 + 5, M - 1, M // 2}:
            if j < M:
                S[b, int(torch.randint(N, (1,), generator=g)), j] = 1.0 + j / M
        for i in {0, 32 * 63 + 1, 32 * 64, N - 1, N // 3}:
            if i < N:
                S[b, i, int(torch.randint(M, (1,), generator=g))] = -0.5 - i / N
    flags = torch.as_tensor(_flags_ref(S), device="cuda")
    got = _grad(X, Y, S, flags)
    dense = _grad(X, Y, S, None)
    for a, b in zip(got, dense):
        assert torch.equal(a, b)
    # against float64
    Xd, Yd, Sd = X.double(), Y.double(), S.double()
    dXr = -2 * Sd @ Yd + 2 * Xd * Sd.sum(2, keepdim=True)
    dYr = -2 * Sd.transpose(1, 2) @ Xd + 2 * Yd * Sd.sum(1)[..., None]
    torch.testing.assert_close(got[0].double(), dXr, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(got[1].double(), dYr, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_features_backward_entry_matches_the_op(dtype):
    """tw_sdtw_features_backward_* (backward + chain rule in one C-ABI call)
    against the soft-DTW op's own backward on the same inputs."""
    import torchwarp_b200 as tw
    B, N, M, D, gamma = 2, 150, 200, 64, 0.05
    X, Y = (t.to(dtype) for t in _inputs(B, N, M, D, 14))
    Xg = X.clone().requires_grad_(True)
    Yg = Y.clone().requires_grad_(True)
    tw.functional.soft_dtw(Xg, Yg, gamma=gamma).sum().backward()
    from torchwarp_b200.udtw import _ops
    out, saved, mask = _ops.sdtw_fused(X, Y, gamma, 0.0)
    lib = nat.lib()
    es = X.element_size()
    wb = lib.tw_sdtw_features_workspace_bytes(B, N, M, es)
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    dX, dY = torch.empty_like(X), torch.empty_like(Y)
    g = torch.ones(B, dtype=dtype, device="cuda")
    fn = getattr(lib, "tw_sdtw_features_backward_" + nat.suffix(dtype))
    nat.check(fn(nat.ptr(X), nat.ptr(Y), nat.ptr(mask), nat.ptr(g), B, N, M, D, gamma,
                 nat.ptr(saved), saved.numel(), nat.ptr(dX), nat.ptr(dY), nat.ptr(ws), wb,
                 nat.stream_of(X)), "tw_sdtw_features_backward")
    torch.cuda.synchronize()
    assert torch.equal(dX, Xg.grad)
    assert torch.equal(dY, Yg.grad)
    assert lib.tw_sdtw_features_workspace_bytes(0, N, M, es) == 0


DP_CASES = [  # B, N, M, gamma, penalty, bandwidth, dtype
    (8, 256, 256, 0.01, False, None, torch.float32),
    (8, 256, 256, 0.01, True, None, torch.float32),
    (3, 300, 520, 0.1, False, None, torch.float32),
    (2, 1024, 1024, 0.01, False, None, torch.float32),   # band groups (few pairs)
    (4, 200, 200, 1.0, True, None, torch.float32),
    (4, 160, 200, 0.05, False, 40, torch.float32),
    (5, 97, 130, 0.01, True, None, torch.float64),
    (3, 64, 300, 0.01, False, None, torch.float64),
]


@pytest.mark.parametrize("case", DP_CASES)
def test_dp_backward_zero_blocks_equal_full_evaluation(case, monkeypatch):
    """The DP backward takes a shortcut through blocks of steps whose
    adjoints are all zero; TW_DP_ALL_BLOCKS=1 evaluates them in full.  Both
    must give the same dL/dcost and dL/dpenalty."""
    import torchwarp_b200 as tw
    B, N, M, gamma, pen, bw, dtype = case
    g = torch.Generator(device="cuda").manual_seed(21)
    C = (torch.rand(B, N, M, device="cuda", generator=g) * 4).to(dtype)
    P = torch.randn(B, N, M, device="cuda", generator=g).to(dtype) if pen else None
    w = torch.linspace(0.5, 2.0, B, device="cuda", dtype=dtype)

    def grads():
        c = C.clone().requires_grad_(True)
        if pen:
            p = P.clone().requires_grad_(True)
            out = tw.functional.udtw_from_cost(c, p, gamma=gamma, bandwidth=bw)
            ((out.distance * w).sum() + (out.penalty * w).sum()).backward()
            return c.grad, p.grad
        d = tw.functional.soft_dtw_from_cost(c, gamma=gamma, bandwidth=bw)
        (d * w).sum().backward()
        return (c.grad,)

    monkeypatch.delenv("TW_DP_ALL_BLOCKS", raising=False)
    fast = grads()
    monkeypatch.setenv("TW_DP_ALL_BLOCKS", "1")
    full = grads()
    for a, b in zip(fast, full):
        assert torch.equal(a, b)
    if gamma <= 0.01 and not pen:
        # most of dL/dcost is exactly zero there, which is what the shortcut uses
        assert (fast[0] == 0).float().mean() > 0.5


def _nz_ref(S):
    """Words [B][ceil(M/32)][4 ceil(N/4)] with bit j & 31 of word [b][j >> 5][i]
    set where S[b, i, j] != 0."""
    B, N, M = S.shape
    mw, npad = -(-M // 32), (N + 3) // 4 * 4
    nz = np.zeros((B, npad, mw * 32), np.uint64)
    nz[:, :N, :M] = (S != 0).cpu().numpy()
    w = (nz.reshape(B, npad, mw, 32) << np.arange(32, dtype=np.uint64)).sum(-1)
    return w.transpose(0, 2, 1).astype(np.uint32)


def _sparse_backward(X, Y, gamma):
    lib = nat.lib()
    B, N, _ = X.shape
    M = Y.shape[1]
    mask, saved, ws = _forward(X, Y, gamma)
    g = torch.linspace(0.5, 1.5, B, device="cuda")
    dC = torch.full((B, N, M), float("nan"), device="cuda")   # unwritten cells stay NaN
    nzm = torch.full_like(mask, -1)                            # zeroed by the call
    fb = lib.tw_sdtw_chunk_flags_bytes(B, N, M)
    flags = torch.full((fb,), 7, dtype=torch.uint8, device="cuda")
    assert lib.tw_sdtw_nonzero_mask_bytes(B, N, M) == nzm.numel() * 4
    nat.check(lib.tw_sdtw_backward_sparse_f32(nat.ptr(g), B, N, M, float(gamma), nat.ptr(saved),
                                              saved.numel(), nat.ptr(mask), nat.ptr(dC),
                                              nat.ptr(nzm), nat.ptr(flags), fb, nat.ptr(ws),
                                              ws.numel(), nat.stream_of(X)), "backward_sparse")
    torch.cuda.synchronize()
    return dC, nzm, flags


SPARSE_CASES = CASES + [(2, 70, 45, 8, 0.01), (2, 66, 90, 64, 0.05)]


@pytest.mark.parametrize("case", SPARSE_CASES)
def test_sparse_backward_writes_the_nonzero_tiles(case):
    """tw_sdtw_backward_sparse_f32: the bit mask marks exactly the nonzero
    values of the dense dL/dcost, those cells hold its values, and the chunk
    flags are those of the dense dL/dcost."""
    B, N, M, D, gamma = case
    X, Y = _inputs(B, N, M, D, 15)
    dense, _ = _backward(X, Y, gamma, flagged=False)
    dC, nzm, flags = _sparse_backward(X, Y, gamma)
    want = _nz_ref(dense)
    np.testing.assert_array_equal(nzm.cpu().numpy().view(np.uint32), want)
    on = dense != 0
    assert torch.equal(dC[on], dense[on])
    np.testing.assert_array_equal(flags.cpu().numpy(), _flags_ref(dense))


@pytest.mark.parametrize("case", SPARSE_CASES)
def test_sparse_chain_rule_equals_dense(case, monkeypatch):
    """The sparse pair (cells outside the mask left NaN) gives the gradients
    of the dense dL/dcost bit for bit, with and without chunk skipping."""
    B, N, M, D, gamma = case
    X, Y = _inputs(B, N, M, D, 16)
    dense, _ = _backward(X, Y, gamma, flagged=False)
    dC, nzm, flags = _sparse_backward(X, Y, gamma)
    want = _grad(X, Y, dense, None)
    for env in (None, "1"):
        if env is None:
            monkeypatch.delenv("TW_GRAD_DENSE", raising=False)
        else:
            monkeypatch.setenv("TW_GRAD_DENSE", env)
        dX, dY = torch.empty_like(X), torch.empty_like(Y)
        nat.check(nat.lib().tw_sqeuclid_grad_sparse_f32(
            nat.ptr(X), nat.ptr(Y), nat.ptr(nzm), nat.ptr(dC), nat.ptr(flags), B, N, M, D,
            nat.ptr(dX), nat.ptr(dY), nat.stream_of(X)), "grad_sparse")
        torch.cuda.synchronize()
        assert torch.isfinite(dX).all() and torch.isfinite(dY).all()
        assert torch.equal(dX, want[0])
        assert torch.equal(dY, want[1])


UDTW_CASES = [  # B, N, M, D, gamma
    (3, 256, 256, 64, 0.01),
    (2, 200, 300, 64, 0.05),
    (2, 160, 192, 64, 1.0),
    (2, 130, 140, 128, 0.01),
    (1, 70, 45, 8, 0.01),      # SIMT chain rule (flags ignored)
]


@pytest.mark.parametrize("case", UDTW_CASES)
def test_udtw_flagged_backward_and_chain_rule_equal_dense(case, monkeypatch):
    """uDTW on features: tw_sdtw_backward_flags_f32 flags the chunks where dL/dcost or
    dL/dpenalty is nonzero, and tw_udtw_features_grad_flagged_f32 gives the dense
    chain rule's dX, dY, dvx, dvy bit for bit."""
    lib = nat.lib()
    B, N, M, D, gamma = case
    X, Y = _inputs(B, N, M, D, 17)
    g = torch.Generator(device="cuda").manual_seed(18)
    vx = 0.25 + torch.rand(B, N, device="cuda", generator=g)
    vy = 0.25 + torch.rand(B, M, device="cuda", generator=g)
    beta, eps = 0.7, 1e-8
    C = torch.empty(B, N, M, device="cuda")
    Q = torch.empty(B, N, M, device="cuda")
    st = nat.stream_of(X)
    nat.check(lib.tw_udtw_cost_f32(nat.ptr(X), nat.ptr(Y), nat.ptr(vx), nat.ptr(vy), B, N, M, D,
                                   beta, eps, nat.ptr(C), nat.ptr(Q), st), "cost")
    sb = lib.tw_sdtw_saved_bytes(B, N, M, 4, 1)
    wb = lib.tw_sdtw_workspace_bytes(B, N, M, 4, 1)
    saved = torch.empty(sb, dtype=torch.uint8, device="cuda")
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    out_r, out_p = torch.empty(B, device="cuda"), torch.empty(B, device="cuda")
    nat.check(lib.tw_sdtw_forward_f32(nat.ptr(C), nat.ptr(Q), B, N, M, float(gamma), 0.0,
                                      nat.ptr(out_r), nat.ptr(out_p), nat.ptr(saved), sb,
                                      nat.ptr(ws), wb, st), "forward")
    gr = torch.linspace(0.5, 1.5, B, device="cuda")
    gp = torch.linspace(1.0, 2.0, B, device="cuda")
    dC0, dQ0 = torch.empty_like(C), torch.empty_like(C)
    nat.check(lib.tw_sdtw_backward_f32(nat.ptr(gr), nat.ptr(gp), B, N, M, float(gamma), 1,
                                       nat.ptr(saved), sb, nat.ptr(dC0), nat.ptr(dQ0),
                                       nat.ptr(ws), wb, st), "backward")
    dC, dQ = torch.empty_like(C), torch.empty_like(C)
    fb = lib.tw_sdtw_chunk_flags_bytes(B, N, M)
    flags = torch.full((fb,), 7, dtype=torch.uint8, device="cuda")
    nat.check(lib.tw_sdtw_backward_flags_f32(nat.ptr(gr), nat.ptr(gp), B, N, M, float(gamma), 1,
                                             nat.ptr(saved), sb, nat.ptr(dC), nat.ptr(dQ),
                                             nat.ptr(flags), fb, nat.ptr(ws), wb, st),
              "backward_flags")
    torch.cuda.synchronize()
    assert torch.equal(dC, dC0) and torch.equal(dQ, dQ0)
    np.testing.assert_array_equal(flags.cpu().numpy(), _flags_ref((dC0 != 0) | (dQ0 != 0)))

    def grads(flagged):
        outs = [torch.empty_like(X), torch.empty_like(Y), torch.zeros_like(vx),
                torch.zeros_like(vy)]
        args = [nat.ptr(X), nat.ptr(Y), nat.ptr(vx), nat.ptr(vy), nat.ptr(C), nat.ptr(dC),
                nat.ptr(dQ)]
        tail = [B, N, M, D, beta, eps] + [nat.ptr(o) for o in outs] + [st]
        if flagged:
            nat.check(lib.tw_udtw_features_grad_flagged_f32(*args, nat.ptr(flags), *tail), "fl")
        else:
            nat.check(lib.tw_udtw_features_grad_f32(*args, *tail), "dense")
        torch.cuda.synchronize()
        return outs

    monkeypatch.delenv("TW_GRAD_DENSE", raising=False)
    for a, b in zip(grads(True), grads(False)):
        assert torch.equal(a, b)
