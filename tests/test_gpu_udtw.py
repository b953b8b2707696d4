"""uDTW / soft-DTW native kernels vs the reference's golden vectors and the oracle (B200).

float64 cases are held to the reference tests' tolerances (atol 1e-10,
rtol 1e-9: tests/test_udtw.py:39-41 of hibana2077/torchwarp).  float32 is
held to the reference's own float32 accuracy bar (max-normalised error vs
the float64 truth < 1e-3, tests/test_udtw.py:125-136).
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


def _run_udtw(tw, inputs, dtype=torch.float64, **kw):
    xs = [_t(x, dtype).requires_grad_(True) for x in inputs]
    d, p = tw.UDTW(**kw)(*xs)
    (d.sum() + 2.0 * p.sum()).backward()
    return [d, p] + [x.grad for x in xs]


@pytest.mark.parametrize("N,M", G.UDTW_SHAPES)
@pytest.mark.parametrize("gamma", G.GAMMAS)
@pytest.mark.parametrize("normalize", [False, True])
def test_udtw_golden(tw, N, M, gamma, normalize):
    ref = G.official("udtw.matches", N=N, M=M, gamma=gamma, normalize=normalize)
    got = _run_udtw(tw, ref["inputs"], gamma=gamma, beta=0.7, normalize=normalize)
    for a, b in zip(got, ref["outputs"]):
        _close(a, b)


@pytest.mark.parametrize("N,M,bandwidth", G.UDTW_BANDS)
def test_udtw_bandwidth_golden(tw, N, M, bandwidth):
    ref = G.official("udtw.bandwidth", N=N, M=M, bandwidth=bandwidth)
    got = _run_udtw(tw, ref["inputs"], gamma=0.1, beta=0.7, bandwidth=bandwidth)
    for a, b in zip(got, ref["outputs"]):
        _close(a, b)


@pytest.mark.parametrize("beta", G.UDTW_BETAS)
def test_udtw_beta_golden(tw, beta):
    ref = G.official("udtw.beta", beta=beta)
    for a, b in zip(_run_udtw(tw, ref["inputs"], gamma=0.1, beta=beta), ref["outputs"]):
        _close(a, b)


def test_udtw_large_golden(tw):
    ref = G.official("udtw.large", B=2, N=40, M=50)
    for a, b in zip(_run_udtw(tw, ref["inputs"], gamma=0.1, beta=0.7), ref["outputs"]):
        _close(a, b)


def test_udtw_float32_accuracy(tw):
    ref = G.official("udtw.float32")
    got = _run_udtw(tw, ref["inputs"], dtype=torch.float32, gamma=0.1, beta=0.7)
    for a, b in zip(got, ref["outputs"]):
        err = np.abs(a.detach().double().cpu().numpy() - b).max() / np.abs(b).max()
        assert err < 1e-3, err


def test_udtw_diff_method_matches_gemm(tw):
    ref = G.official("udtw.large", B=2, N=40, M=50)
    a = _run_udtw(tw, ref["inputs"], gamma=0.1, beta=0.7, method="gemm")
    b = _run_udtw(tw, ref["inputs"], gamma=0.1, beta=0.7, method="diff")
    for x, y in zip(a, b):
        _close(x, y.detach().cpu().numpy())


@pytest.mark.parametrize("T,U", G.SDTW_SHAPES)
@pytest.mark.parametrize("gamma", G.GAMMAS)
def test_soft_dtw_cost_golden(tw, T, U, gamma):
    ref = G.official("jeanie.soft_dtw", T=T, U=U, gamma=gamma)
    c = _t(ref["cost"][None]).requires_grad_(True)
    d = tw.functional.soft_dtw_from_cost(c, gamma=gamma)
    d.sum().backward()
    _close(d[0], ref["value"])
    _close(c.grad[0], ref["grad"])


def test_soft_dtw_cost_large_golden(tw):
    ref = G.official("jeanie.large", name="soft_dtw", shape=(60, 70))
    c = _t(ref["cost"][None]).requires_grad_(True)
    d = tw.functional.soft_dtw_from_cost(c, gamma=0.1)
    d.sum().backward()
    _close(d[0], ref["value"])
    _close(c.grad[0], ref["grad"])


SCALED = ["udtw_cfg1", "udtw_band", "udtw_norm", "udtw_nm", "sdtw_cfg2", "sdtw_cfg5",
          "sdtw_norm", "sdtw_cost_band", "sdtw_cost_long"]


@pytest.mark.parametrize("name", SCALED)
def test_scaled_reference_backend(tw, name):
    """Config-shaped cases against the reference's float64 PyTorch backend."""
    ins, kw, vals, grads = G.scaled(name)
    xs = [_t(x).requires_grad_(True) for x in ins]
    if name.startswith("udtw"):
        d, p = tw.functional.udtw(*xs, **kw)
        (d.sum() + 2.0 * p.sum()).backward()
        got_v = [d, p]
    elif name.startswith("sdtw_cost"):
        d = tw.functional.soft_dtw_from_cost(xs[0], **kw)
        d.sum().backward()
        got_v = [d]
    else:
        d = tw.functional.soft_dtw(xs[0], xs[1], **kw)
        d.sum().backward()
        got_v = [d]
    for a, b in zip(got_v, vals):
        _close(a, b)
    for x, g in zip(xs, grads):
        _close(x.grad, g, atol=1e-9, rtol=1e-8)


@pytest.mark.parametrize("B,N,M,band", [
    (1, 1, 1, 0), (3, 1, 9, 0), (3, 9, 1, 0), (5, 33, 7, 0), (4, 31, 32, 0), (2, 64, 65, 0),
    (7, 65, 64, 0), (2, 129, 140, 0), (3, 200, 260, 0), (300, 17, 23, 0), (611, 40, 41, 0),
    (2, 150, 160, 12), (3, 96, 100, 5.5), (700, 70, 60, 0), (650, 100, 95, 9),
    (3000, 64, 20, 0), (2600, 128, 12, 0), (2700, 96, 10, 0),
])
def test_dp_vs_oracle(tw, orc, B, N, M, band):
    """Shapes that cross the sub-band, band-pass and pairs-per-warp boundaries."""
    g = torch.Generator().manual_seed(B * 1000 + N * 10 + M)
    C = torch.rand(B, N, M, generator=g, dtype=torch.float64)
    Q = torch.randn(B, N, M, generator=g, dtype=torch.float64)
    gr = torch.rand(B, generator=g, dtype=torch.float64)
    gp = torch.randn(B, generator=g, dtype=torch.float64)
    c, q = C.to(DEV).requires_grad_(True), Q.to(DEV).requires_grad_(True)
    d, p = tw.functional.udtw_from_cost(c, q, gamma=0.3, bandwidth=band or None)
    (d * gr.to(DEV) + p * gp.to(DEV)).sum().backward()
    od, op, dC, dQ = orc.udtw_from_cost(C.numpy(), Q.numpy(), gamma=0.3, bandwidth=band or None,
                                        g_d=gr.numpy(), g_p=gp.numpy())
    _close(d, od)
    _close(p, op)
    _close(c.grad, dC)
    _close(q.grad, dQ)


@pytest.mark.parametrize("B,N,M", [(4, 250, 300), (33, 128, 1024), (700, 70, 90)])
def test_soft_dtw_cost_vs_oracle(tw, orc, B, N, M):
    g = torch.Generator().manual_seed(N + M)
    C = torch.rand(B, N, M, generator=g, dtype=torch.float64)
    c = C.to(DEV).requires_grad_(True)
    d = tw.functional.soft_dtw_from_cost(c, gamma=0.05)
    d.sum().backward()
    od, dC = orc.soft_dtw_from_cost(C.numpy(), gamma=0.05)
    _close(d, od)
    _close(c.grad, dC)


@pytest.mark.parametrize("ks", [1, 2, 3, 4])
@pytest.mark.parametrize("B,N,M,pen", [
    (3, 200, 260, False), (2, 129, 300, True), (2, 256, 520, False), (70, 100, 95, True),
    (5, 384, 130, False),
])
def test_sub_band_counts_vs_oracle(tw, orc, monkeypatch, ks, B, N, M, pen):
    """Every sub-band count the plan can choose (forced through TW_STREAM_KS),
    float64, with and without the uDTW penalty stream."""
    monkeypatch.setenv("TW_STREAM_KS", str(ks))
    g = torch.Generator().manual_seed(ks * 7919 + B * 31 + N + M)
    C = torch.rand(B, N, M, generator=g, dtype=torch.float64)
    gr = torch.rand(B, generator=g, dtype=torch.float64)
    c = C.to(DEV).requires_grad_(True)
    if pen:
        Q = torch.randn(B, N, M, generator=g, dtype=torch.float64)
        gp = torch.randn(B, generator=g, dtype=torch.float64)
        q = Q.to(DEV).requires_grad_(True)
        d, p = tw.functional.udtw_from_cost(c, q, gamma=0.3)
        (d * gr.to(DEV) + p * gp.to(DEV)).sum().backward()
        od, op, dC, dQ = orc.udtw_from_cost(C.numpy(), Q.numpy(), gamma=0.3, g_d=gr.numpy(),
                                            g_p=gp.numpy())
        _close(p, op)
        _close(q.grad, dQ)
    else:
        d = tw.functional.soft_dtw_from_cost(c, gamma=0.3)
        (d * gr.to(DEV)).sum().backward()
        od, dC = orc.soft_dtw_from_cost(C.numpy(), gamma=0.3)
        dC = dC * gr.numpy()[:, None, None]
    _close(d, od)
    _close(c.grad, dC)


@pytest.mark.parametrize("G,ks,B,N,M,pen,band", [
    (2, 2, 3, 256, 300, False, 0),      # N a multiple of the band height: seed from below
    (4, 2, 3, 256, 300, True, 0),
    (4, 1, 5, 250, 310, True, 0),       # ragged last band
    (2, 1, 5, 250, 310, False, 0),
    (4, 4, 2, 1024, 40, False, 0),      # L padded to G (32 KS + 128)
    (2, 2, 2, 200, 200, True, 15),      # Sakoe-Chiba band
    (4, 1, 2999, 128, 20, True, 0),     # several pairs per group, ragged split
    (2, 2, 1000, 256, 260, False, 4.5),
    # g * D not a multiple of 32: the per-lane rings are indexed by step, not column
    (2, 2, 3, 256, 1030, False, 0),     # L = 1040, D = 520
    (4, 2, 2, 512, 1100, True, 0),      # L = 1120, D = 280
    (4, 1, 3, 256, 700, True, 0),       # L = 704, D = 176
    (4, 4, 2, 1024, 1030, False, 40),   # L = 1056, D = 264
])
def test_band_groups_vs_oracle(tw, orc, monkeypatch, G, ks, B, N, M, pen, band):
    """Band groups (TW_STREAM_G): G warps per pair set, one band in G each,
    float64 against the oracle, and no device-side wait ran out."""
    monkeypatch.setenv("TW_STREAM_G", str(G))
    monkeypatch.setenv("TW_STREAM_KS", str(ks))
    g = torch.Generator().manual_seed(G * 101 + ks * 7 + B + N + M)
    C = torch.rand(B, N, M, generator=g, dtype=torch.float64)
    Q = torch.randn(B, N, M, generator=g, dtype=torch.float64) if pen else np.zeros((B, N, M))
    gr = torch.rand(B, generator=g, dtype=torch.float64)
    gp = torch.randn(B, generator=g, dtype=torch.float64)
    c = C.to(DEV).requires_grad_(True)
    bw = band or None
    if pen:
        q = Q.to(DEV).requires_grad_(True)
        d, p = tw.functional.udtw_from_cost(c, q, gamma=0.3, bandwidth=bw)
        (d * gr.to(DEV) + p * gp.to(DEV)).sum().backward()
        od, op, dC, dQ = orc.udtw_from_cost(C.numpy(), Q.numpy(), gamma=0.3, bandwidth=bw,
                                            g_d=gr.numpy(), g_p=gp.numpy())
        _close(p, op)
        _close(q.grad, dQ)
    else:
        d = tw.functional.soft_dtw_from_cost(c, gamma=0.3, bandwidth=bw)
        (d * gr.to(DEV)).sum().backward()
        od, _, dC, _ = orc.udtw_from_cost(C.numpy(), Q, gamma=0.3, bandwidth=bw, g_d=gr.numpy())
    _close(d, od)
    _close(c.grad, dC)
    assert tw._native.lib().tw_device_error() == 0


@pytest.mark.parametrize("ks", [2, 4])
def test_band_groups_agree_fp32(tw, monkeypatch, ks):
    """Splitting a pair's bands over 1, 2 or 4 warps does not change the
    arithmetic of any cell: float32 values are bit-identical."""
    g = torch.Generator().manual_seed(12)
    C = torch.rand(6, 512, 1100, generator=g).to(DEV)  # 8 or 4 bands: G = 4 applies
    monkeypatch.setenv("TW_STREAM_KS", str(ks))
    out = []
    for G in (1, 2, 4):
        monkeypatch.setenv("TW_STREAM_G", str(G))
        c = C.clone().requires_grad_(True)
        d = tw.functional.soft_dtw_from_cost(c, gamma=0.1)
        d.sum().backward()
        out.append((d.detach(), c.grad))
    for d, gC in out[1:]:
        assert torch.equal(d, out[0][0])
        torch.testing.assert_close(gC, out[0][1], rtol=1e-6, atol=1e-9)
    assert tw._native.lib().tw_device_error() == 0


def _saved_bytes(tw, B, N, M, eb, pen):
    return tw._native.lib().tw_sdtw_saved_bytes(B, N, M, eb, int(pen))


@pytest.mark.parametrize("B,N,M,eb,pen,ks,G", [
    (512, 1024, 1024, 4, False, 2, 4),    # 3.5 pairs per SM: 4 warps per pair
    (1184, 1024, 1024, 4, False, 2, 2),
    (1775, 1024, 1024, 4, False, 2, 2),   # just under 12 pairs per SM
    (1776, 1024, 1024, 4, False, 2, 1),
    (4096, 1024, 1024, 4, False, 2, 1),
    (512, 1024, 1024, 8, False, 2, 4),    # fp64 too
    (512, 200, 200, 4, False, 2, 1),      # M + 1 < 2 (64 + 128): no group
    (512, 640, 1024, 4, False, 2, 2),     # 10 bands: G = 4 does not divide
    (512, 576, 1024, 4, False, 2, 1),     # 9 bands: no group
    (512, 1000, 300, 4, False, 2, 1),     # M + 1 < 384
    (512, 1024, 1024, 4, True, 1, 4),     # uDTW: one sub-band, 4 warps per pair
    (2048, 1024, 1024, 4, True, 1, 1),
])
def test_sub_band_choice(tw, monkeypatch, B, N, M, eb, pen, ks, G):
    """The plan's default sub-band count and band-group size, read through the
    saved-stream size (which depends on both) against the size with both
    forced."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if sms != 148:
        pytest.skip("thresholds are written for 148 SMs")
    monkeypatch.delenv("TW_STREAM_KS", raising=False)
    monkeypatch.delenv("TW_STREAM_G", raising=False)
    auto = _saved_bytes(tw, B, N, M, eb, pen)
    monkeypatch.setenv("TW_STREAM_KS", str(ks))
    monkeypatch.setenv("TW_STREAM_G", str(G))
    assert auto == _saved_bytes(tw, B, N, M, eb, pen)
    # the size tells the choices apart
    monkeypatch.setenv("TW_STREAM_KS", str(1 if ks == 2 else 2))
    assert auto != _saved_bytes(tw, B, N, M, eb, pen)


def test_sub_band_counts_agree_fp32(tw, monkeypatch):
    """The soft-min recursion per cell does not depend on how rows are split
    into bands, so 2 and 4 sub-bands give bit-identical values and gradients."""
    g = torch.Generator().manual_seed(11)
    C = torch.rand(6, 640, 700, generator=g).to(DEV)
    out = []
    for ks in (2, 4):
        monkeypatch.setenv("TW_STREAM_KS", str(ks))
        c = C.clone().requires_grad_(True)
        d = tw.functional.soft_dtw_from_cost(c, gamma=0.1)
        d.sum().backward()
        out.append((d.detach(), c.grad))
    assert torch.equal(out[0][0], out[1][0])
    torch.testing.assert_close(out[0][1], out[1][1], rtol=1e-6, atol=1e-9)


def test_soft_dtw_features_fp32_vs_fp64(tw, orc):
    """cfg5-shaped soft-DTW (N=M=1024, D=64, gamma=0.01) in float32 against
    the float64 oracle: the forward value within 1e-5 relative."""
    g = torch.Generator().manual_seed(5)
    X = torch.randn(2, 1024, 64, generator=g, dtype=torch.float64)
    Y = torch.randn(2, 1024, 64, generator=g, dtype=torch.float64)
    x = X.float().to(DEV).requires_grad_(True)
    d = tw.functional.soft_dtw(x, Y.float().to(DEV), gamma=0.01)
    d.sum().backward()
    od, odx, _ = orc.soft_dtw(X.float().double().numpy(), Y.float().double().numpy(), gamma=0.01)
    rel = np.abs(d.detach().double().cpu().numpy() - od) / np.abs(od)
    assert rel.max() < 1e-5, rel
    assert torch.isfinite(x.grad).all()


def test_bitwise_deterministic(tw):
    g = torch.Generator().manual_seed(11)
    X = torch.randn(64, 300, 16, generator=g).to(DEV)
    Y = torch.randn(64, 280, 16, generator=g).to(DEV)
    S = (torch.rand(64, 300, 1, generator=g) + 0.5).to(DEV)
    T = (torch.rand(64, 280, 1, generator=g) + 0.5).to(DEV)

    def run():
        xs = [t.clone().requires_grad_(True) for t in (X, Y, S, T)]
        d, p = tw.UDTW(gamma=0.1, beta=0.7)(*xs)
        (d.sum() + p.sum()).backward()
        return [d.detach(), p.detach()] + [t.grad for t in xs]

    first = run()
    for _ in range(2):
        assert all(torch.equal(a, b) for a, b in zip(run(), first))


def test_unreachable_band_raises(tw):
    g = torch.Generator().manual_seed(0)
    xs = [torch.rand(1, 3, 5, generator=g), torch.rand(1, 9, 5, generator=g),
          torch.rand(1, 3, 1, generator=g) + 0.5, torch.rand(1, 9, 1, generator=g) + 0.5]
    with pytest.raises(ValueError):
        tw.UDTW(gamma=0.1, bandwidth=2)(*[x.to(DEV) for x in xs])


def test_cpu_tensors_rejected(tw):
    with pytest.raises(RuntimeError, match="CUDA"):
        tw.functional.soft_dtw_from_cost(torch.rand(1, 3, 4), gamma=0.1)


def _unpack_mask(mask, N, M):
    """[B, ceil(M/32), NP] int32 words -> [B, N, M] bool (bit j & 31 of word j >> 5)."""
    w = mask.to(torch.int64) & 0xFFFFFFFF
    j = torch.arange(M, device=mask.device)
    bits = (w[:, j // 32, :N] >> (j % 32)[None, :, None]) & 1
    return bits.transpose(1, 2).bool().contiguous()


@pytest.mark.parametrize("shape", [(3, 70, 45), (2, 200, 130), (5, 33, 64), (4, 1, 1),
                                   (2, 129, 300), (1, 257, 9), (2, 70, 40), (1, 100, 296)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("ks,G", [(None, None), (3, None), (4, None), (1, 4), (2, 2)])
def test_sdtw_backward_masked(tw, monkeypatch, shape, dtype, ks, G):
    """tw_sdtw_backward_masked writes the plain backward's d_cost with the
    cells whose mask bit is clear set to zero, bit for bit (with the plan's
    own sub-band count, with 3 and 4 forced, and with band groups)."""
    if ks is not None:
        monkeypatch.setenv("TW_STREAM_KS", str(ks))
    if G is not None:
        monkeypatch.setenv("TW_STREAM_G", str(G))
    from torchwarp_b200 import _native as nat
    from torchwarp_b200.udtw import _ops
    B, N, M = shape
    g = torch.Generator().manual_seed(N * 7 + M)
    C = torch.rand(B, N, M, generator=g, dtype=torch.float64).to(DEV, dtype)
    mask = torch.randint(-2 ** 31, 2 ** 31, (B, (M + 31) // 32, (N + 3) // 4 * 4), generator=g,
                         dtype=torch.int64).to(torch.int32).to(DEV)
    gamma = 0.1
    out_r, _, saved = _ops._dp_forward(C, None, gamma, 0.0)
    grad_r = torch.rand(B, generator=g, dtype=torch.float64).to(DEV, dtype) + 0.5
    d_cost, _ = _ops._dp_backward(saved, grad_r, grad_r, N, M, gamma, False)
    s_cost = torch.full_like(d_cost, float("nan"))
    wb = _ops._ws_bytes(B, N, M, dtype, False)
    ws = torch.empty(wb, dtype=torch.uint8, device=DEV)
    fn = getattr(nat.lib(), "tw_sdtw_backward_masked_" + nat.suffix(dtype))
    nat.check(fn(nat.ptr(grad_r), B, N, M, gamma, nat.ptr(saved), saved.numel(), nat.ptr(mask),
                 nat.ptr(s_cost), nat.ptr(ws), wb, nat.stream_of(C)), "tw_sdtw_backward_masked")
    torch.cuda.synchronize()
    want = torch.where(_unpack_mask(mask, N, M), d_cost, torch.zeros_like(d_cost))
    assert torch.equal(s_cost, want)
