"""Public cost builders on the tensor cores (B200).

``squared_euclidean_cost`` and ``euclidean_cost`` (hibana2077/torchwarp
src/torchwarp/jeanie/distances.py:15-38) run the |q|^2 + |s|^2 - 2 q.s
contraction on tcgen05 (3xTF32, fp32 accumulate) when it is a real dense
contraction: float32, 64 <= D <= 256, at least 64 query rows and 32 support
frames, D and the frame count multiples of 4.  Both layouts are covered (two
sequences [B, N, D] x [B, M, D]; query/support [B, K, T, D] x [B, U, D]),
values and gradients against the float64 formula, and agreement with the
SIMT kernels (``TW_COST_SIMT=1``).  (The zero-distance convention, no
gradient through sqrt at 0, is the same code as on the SIMT path; a GEMM-form
distance of two equal frames is a rounding residue, not an exact 0, in any
implementation, so it is not a meaningful parity case here.)
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def tw():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torchwarp_b200
    return torchwarp_b200


def _ref_cost(q, s, euclid):
    """float64 formula; the Euclidean root has zero gradient at 0."""
    bq = q.ndim > s.ndim
    sp = s.unsqueeze(-3) if bq else s
    sq = ((q * q).sum(-1)[..., :, None] + (sp * sp).sum(-1)[..., None, :]
          - 2.0 * q @ sp.transpose(-1, -2)).clamp_min(0)
    if not euclid:
        return sq
    pos = sq > 0
    return torch.where(pos, torch.sqrt(torch.where(pos, sq, torch.ones_like(sq))),
                       torch.zeros_like(sq))


CASES = [
    ("two_seq_d64", (3, 200, 64), (3, 160, 64)),
    ("two_seq_d256", (2, 130, 256), (2, 96, 256)),
    ("query_support_d128", (2, 4, 40, 128), (2, 64, 128)),
]


@pytest.mark.parametrize("euclid", [False, True], ids=["sqeuclidean", "euclidean"])
@pytest.mark.parametrize("name,qshape,sshape", CASES, ids=[c[0] for c in CASES])
def test_cost_and_grad_tensor_core(tw, name, qshape, sshape, euclid):
    g = torch.Generator().manual_seed(hash(name) % 1000)
    q = torch.randn(*qshape, generator=g, dtype=torch.float64)
    s = torch.randn(*sshape, generator=g, dtype=torch.float64)
    fn = tw.euclidean_cost if euclid else tw.squared_euclidean_cost
    qf = q.float().to(DEV).requires_grad_(True)
    sf = s.float().to(DEV).requires_grad_(True)
    c = fn(qf, sf)
    up = torch.randn(c.shape, generator=g, dtype=torch.float64)
    (c * up.float().to(DEV)).sum().backward()

    qd, sd = q.float().double().requires_grad_(True), s.float().double().requires_grad_(True)
    cd = _ref_cost(qd, sd, euclid)
    (cd * up).sum().backward()
    scale = cd.abs().max()
    assert (c.detach().double().cpu() - cd.detach()).abs().max() / scale < 2e-6
    for got, want in ((qf.grad, qd.grad), (sf.grad, sd.grad)):
        err = (got.double().cpu() - want).abs().max() / want.abs().max()
        assert err < 2e-5, err


def test_tensor_core_agrees_with_simt(tw, monkeypatch):
    g = torch.Generator().manual_seed(9)
    q = torch.randn(2, 256, 64, generator=g).to(DEV)
    s = torch.randn(2, 192, 64, generator=g).to(DEV)
    out = []
    for simt in ("0", "1"):
        monkeypatch.setenv("TW_COST_SIMT", simt)
        a, b = q.clone().requires_grad_(True), s.clone().requires_grad_(True)
        c = tw.euclidean_cost(a, b)
        c.sum().backward()
        out.append((c.detach(), a.grad, b.grad))
    for x, y in zip(*out):
        torch.testing.assert_close(x, y, rtol=1e-5, atol=1e-5)


def test_tensor_core_cost_vmap(tw):
    """vmap over the tensor-core route of euclidean_cost (the qs_cost fold
    rule) matches the flattened batch."""
    g = torch.Generator().manual_seed(10)
    q = torch.randn(2, 3, 96, 64, generator=g).to(DEV)
    s = torch.randn(2, 3, 64, 64, generator=g).to(DEV)
    got = torch.func.vmap(tw.euclidean_cost)(q, s)
    want = tw.euclidean_cost(q.reshape(6, 96, 64), s.reshape(6, 64, 64)).reshape(2, 3, 96, 64)
    torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-5)
