"""Pin the CPU oracle against the reference's golden vectors (no GPU).

Every case below is a stored float64 output of the official uDTW / JEANIE
code (``official.npz``) or of the reference's PyTorch backend at
config-shaped sizes (``scaled.npz``).  Tolerances are the reference tests'
own: atol 1e-10, rtol 1e-9 (tests/test_udtw.py:39-41, tests/test_jeanie.py:23).
"""

import numpy as np
import pytest

import golden_data as G

ATOL, RTOL = 1e-10, 1e-9


def close(a, b, atol=ATOL, rtol=RTOL):
    np.testing.assert_allclose(np.asarray(a), np.asarray(b), atol=atol, rtol=rtol)


def _udtw_check(orc, ref, **kw):
    X, Y, SX, SY = ref["inputs"]
    got = orc.udtw(X, Y, SX, SY, beta=kw.pop("beta", 0.7), g_d=1.0, g_p=2.0, **kw)
    for a, b in zip(got, ref["outputs"]):
        close(a, b)


@pytest.mark.parametrize("N,M", G.UDTW_SHAPES)
@pytest.mark.parametrize("gamma", G.GAMMAS)
@pytest.mark.parametrize("normalize", [False, True])
def test_udtw_matches(orc, N, M, gamma, normalize):
    _udtw_check(orc, G.official("udtw.matches", N=N, M=M, gamma=gamma, normalize=normalize),
                gamma=gamma, normalize=normalize)


@pytest.mark.parametrize("N,M,bandwidth", G.UDTW_BANDS)
def test_udtw_bandwidth(orc, N, M, bandwidth):
    _udtw_check(orc, G.official("udtw.bandwidth", N=N, M=M, bandwidth=bandwidth), gamma=0.1,
                bandwidth=bandwidth)


@pytest.mark.parametrize("beta", G.UDTW_BETAS)
def test_udtw_beta(orc, beta):
    _udtw_check(orc, G.official("udtw.beta", beta=beta), gamma=0.1, beta=beta)


def test_udtw_large_and_float32_truth(orc):
    _udtw_check(orc, G.official("udtw.large", B=2, N=40, M=50), gamma=0.1)
    _udtw_check(orc, G.official("udtw.float32"), gamma=0.1)


def test_pairwise_matrices(orc):
    ref = G.official("udtw.pairwise_matrices")
    X, Y, SX, SY = ref["inputs"]
    cost, pen, _, _, var = orc.udtw_matrices(X, Y, SX[..., 0] ** 2, SY[..., 0] ** 2, 0.5, 1e-8)
    for a, b in zip((cost, pen, var), ref["outputs"]):
        close(a, b, atol=1e-12, rtol=1e-10)


def test_udtw_vmap_values(orc):
    ref = G.official("udtw.vmap")
    for v, scale in enumerate((1.0, 1.1, 0.9)):
        X, Y, SX, SY = (scale * x for x in ref["inputs"])
        d, p, *_ = orc.udtw(X, Y, SX, SY, beta=0.5, gamma=0.3)
        close(d, ref["distance"][v])
        close(p, ref["penalty"][v])


@pytest.mark.parametrize("T,U", G.SDTW_SHAPES)
@pytest.mark.parametrize("gamma", G.GAMMAS)
def test_soft_dtw_cost(orc, T, U, gamma):
    ref = G.official("jeanie.soft_dtw", T=T, U=U, gamma=gamma)
    d, dc = orc.soft_dtw_from_cost(ref["cost"][None], gamma=gamma)
    close(d[0], ref["value"])
    close(dc[0], ref["grad"])


@pytest.mark.parametrize("K,T,U", G.JEANIE_1D_SHAPES)
@pytest.mark.parametrize("shift", G.JEANIE_1D_SHIFTS)
def test_jeanie_1d(orc, K, T, U, shift):
    ref = G.official("jeanie.jeanie_1d", K=K, T=T, U=U, shift=shift)
    d, R, dc = orc.jeanie_from_cost(ref["cost"][None], gamma=0.1, max_shift=shift)
    close(d[0], ref["value"])
    close(dc[0], ref["grad"])
    close(R[0], ref["accumulator"])


@pytest.mark.parametrize("K1,K2,T,U", G.JEANIE_2D_SHAPES)
@pytest.mark.parametrize("s_az,s_alt", G.JEANIE_2D_SHIFTS)
def test_jeanie_2d(orc, K1, K2, T, U, s_az, s_alt):
    ref = G.official("jeanie.jeanie_2d", K1=K1, K2=K2, T=T, U=U, s_az=s_az, s_alt=s_alt)
    d, _, dc = orc.jeanie_from_cost(ref["cost"][None], gamma=0.1, max_shift=(s_az, s_alt))
    close(d[0], ref["value"])
    close(dc[0], ref["grad"])


def test_jeanie_batched(orc):
    ref = G.official("jeanie.batched")
    close(orc.jeanie_from_cost(ref["cost_1d"], gamma=0.1, max_shift=1)[0], ref["value_1d"])
    close(orc.jeanie_from_cost(ref["cost_2d"], gamma=0.1, max_shift=(1, 1))[0], ref["value_2d"])


@pytest.mark.parametrize("name,shape", G.FVM_CASES)
def test_fvm_cost(orc, name, shape):
    ref = G.official("jeanie.fvm", name=name)
    d, dc = orc.fvm_from_cost(ref["cost"][None], gamma=0.1)
    close(d[0], ref["value"])
    close(dc[0], ref["grad"])
    close(orc.fvm_from_cost(ref["batch"], gamma=0.1)[0], ref["batch_value"])


@pytest.mark.parametrize("name,shape,shift", G.LARGE_COST)
def test_large_cost(orc, name, shape, shift):
    ref = G.official("jeanie.large", name=name, shape=shape)
    c = ref["cost"][None]
    if name == "soft_dtw":
        d, dc = orc.soft_dtw_from_cost(c, gamma=0.1)
    elif name.startswith("fvm"):
        d, dc = orc.fvm_from_cost(c, gamma=0.1)
    else:
        d, _, dc = orc.jeanie_from_cost(c, gamma=0.1, max_shift=shift)
    close(d[0], ref["value"])
    close(dc[0], ref["grad"])


@pytest.mark.parametrize("name", G.DISTANCES)
def test_distances(orc, name):
    ref = G.official("jeanie.distance", name=name)
    val, dq, ds = orc.distance(name, ref["q"], ref["s"])
    close(val, ref["value"])
    close(dq, ref["grads"][0])
    close(ds, ref["grads"][1])
    close(orc.distance(name, ref["qb"], ref["sb"])[0], ref["batch_value"])


def test_end_to_end(orc):
    ref = G.official("jeanie.end_to_end")
    d, _, dq, ds = orc.jeanie(ref["q"][None], ref["s"][None], gamma=0.1, max_shift=1)
    close(d[0], ref["value"])
    close(dq[0], ref["grads"][0])
    close(ds[0], ref["grads"][1])


@pytest.mark.parametrize("metric", G.METRICS)
@pytest.mark.parametrize("K,T,U,shift", G.FEATURES_1D)
def test_jeanie_features_1d(orc, metric, K, T, U, shift):
    ref = G.official("jeanie.features_1d", metric=metric, K=K, T=T, U=U, shift=shift)
    d, _, dq, ds = orc.jeanie(ref["q"], ref["s"], gamma=0.1, max_shift=shift, metric=metric)
    close(d, ref["value"])
    close(dq, ref["grads"][0])
    close(ds, ref["grads"][1])


@pytest.mark.parametrize("metric", ["euclidean", "sqeuclidean"])
def test_jeanie_features_2d(orc, metric):
    ref = G.official("jeanie.features_2d", metric=metric)
    d, R, dq, ds = orc.jeanie(ref["q"], ref["s"], gamma=0.1, max_shift=(1, 1), metric=metric)
    close(d, ref["value"])
    close(dq, ref["grads"][0])
    close(ds, ref["grads"][1])
    close(R[0], ref["accumulator"])


@pytest.mark.parametrize("K,T,U,shift", G.ACCUMULATOR_COST)
def test_accumulator_cost(orc, K, T, U, shift):
    ref = G.official("parity.accumulator_cost", K=K, T=T, U=U, shift=shift)
    c = ref["cost"][None]
    _, R, _ = orc.jeanie_from_cost(c, gamma=0.3, max_shift=shift)
    _, _, dc = orc.jeanie_from_cost(c, gamma=0.3, max_shift=shift, g_R=0.1 * 2.0 * R / R.size)
    close(dc[0], ref["grad"])


def test_accumulator_2d(orc):
    ref = G.official("parity.accumulator_2d")
    c = ref["cost"][None]
    _, R, _ = orc.jeanie_from_cost(c, gamma=0.3, max_shift=(1, 1))
    _, _, dc = orc.jeanie_from_cost(c, gamma=0.3, max_shift=(1, 1), g_R=np.cos(R))
    close(dc[0], ref["grad"])


@pytest.mark.parametrize("metric", ["euclidean", "sqeuclidean"])
def test_accumulator_features(orc, metric):
    ref = G.official("parity.accumulator_features", metric=metric)
    q, s = ref["q"][None], ref["s"][None]
    _, R, _, _ = orc.jeanie(q, s, gamma=0.3, max_shift=1, metric=metric)
    _, _, dq, ds = orc.jeanie(q, s, gamma=0.3, max_shift=1, metric=metric,
                              g_R=0.1 * 2.0 * R / R.size)
    close(dq[0], ref["grads"][0])
    close(ds[0], ref["grads"][1])


def test_vmap_values(orc):
    ref = G.official("parity.vmap")
    cost = ref["cost"]
    for v in range(cost.shape[0]):
        close(orc.jeanie_from_cost(cost[v], gamma=0.3, max_shift=1)[0], ref["cost_value"][v])
        q, s = ref["q"][v], ref["s"][v]
        close(orc.jeanie(q, s, gamma=0.3, max_shift=1)[0], ref["features_value"][v])


@pytest.mark.parametrize("name", G.SCALED_CASES)
def test_scaled_cases(orc, name):
    """Config-shaped cases against the reference's own float64 torch backend."""
    ins, kw, vals, grads = G.scaled(name)
    kw = dict(kw)
    if name.startswith("udtw"):
        d, p, *g = orc.udtw(*ins, g_d=1.0, g_p=2.0, **kw)
        got_v, got_g = [d, p], g
    elif name.startswith("sdtw_cost"):
        d, dc = orc.soft_dtw_from_cost(ins[0], **kw)
        got_v, got_g = [d], [dc]
    elif name.startswith("sdtw"):
        d, dx, dy = orc.soft_dtw(ins[0], ins[1], **kw)
        got_v, got_g = [d], [dx, dy]
    elif name.startswith("jeanie_cost"):
        d, _, dc = orc.jeanie_from_cost(ins[0], **kw)
        got_v, got_g = [d], [dc]
    elif name.startswith("jeanie"):
        d, _, dq, ds = orc.jeanie(ins[0], ins[1], **kw)
        got_v, got_g = [d], [dq, ds]
    elif name.startswith("fvm_cost"):
        d, dc = orc.fvm_from_cost(ins[0], **kw)
        got_v, got_g = [d], [dc]
    else:
        d, dq, ds = orc.fvm(ins[0], ins[1], **kw)
        got_v, got_g = [d], [dq, ds]
    for a, b in zip(got_v, vals):
        close(a, b)
    assert len(got_g) == len(grads)
    for a, b in zip(got_g, grads):
        close(a, b, atol=1e-9, rtol=1e-8)


def test_optimal_path_known_answers(orc):
    # exact-DTW path cost equals the summed cost along the argmin path
    # (reference tests/test_paths.py:13-41 restated on a fixed seed)
    rng = np.random.default_rng(0)
    cost = rng.random((9, 12))
    path = orc.optimal_path(cost[None], 0)
    T, U = cost.shape
    R = np.full((T + 1, U + 1), np.inf)
    R[0, 0] = 0
    for t in range(1, T + 1):
        for u in range(1, U + 1):
            R[t, u] = cost[t - 1, u - 1] + min(R[t - 1, u], R[t, u - 1], R[t - 1, u - 1])
    assert path[0][:2] == (0, 0) and path[-1][:2] == (T - 1, U - 1)
    assert abs(sum(cost[t, u] for t, u, _ in path) - R[T, U]) < 1e-12


@pytest.mark.parametrize("name", G.HIGHER_COST_CASES)
def test_oracle_second_order_identity(orc, name):
    """soft-DTW's Hessian-vector product and jvp through the uDTW penalty
    recursion, against the reference's own autograd DP
    (tests/golden/make_higher_order.py).  With penalty Q = V, the uDTW end
    value is <E, V> (E = dd/dC), and its gradient for seeds (0, g) is
    g * (d^2 d/dC^2) V: the identity the native double backward uses."""
    h = G.higher(name)
    gamma, band = h["args"]
    bw = band or None
    d, p, dC, dQ = orc.udtw_from_cost(h["C"], h["V"], gamma=gamma, bandwidth=bw, g_d=0.0,
                                      g_p=h["g"])
    close(d, h["d"])
    close(p, h["hvp_g"], atol=1e-9, rtol=1e-8)
    close(dC, h["hvp_C"], atol=1e-9, rtol=1e-8)
    close(dQ, h["dC"])
    _, jp, _, _ = orc.udtw_from_cost(h["C"], h["T"], gamma=gamma, bandwidth=bw, g_d=1.0, g_p=0.0)
    close(jp, h["jvp"], atol=1e-9, rtol=1e-8)
