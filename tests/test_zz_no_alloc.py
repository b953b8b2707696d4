"""The allocation-free soft-DTW forward entry point, through the C ABI (B200).

tw_sdtw_forward_noalloc_f32 serves callers that own all device memory and can
give the library only its inputs and outputs, never a scratch workspace.  Its
results must match tw_sdtw_forward_f32 (caller workspace) call after call, and
shapes whose scratch would not fit its static buffer must be refused.  This
file runs last so that a failure here leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STATIC_BYTES = 4 << 20
# float32 tolerance of the other GPU tests (forward values within 1e-5
# relative); the two entry points run the same kernel, so far tighter holds.
RTOL, ATOL = 1e-6, 1e-7


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from torchwarp_b200 import _native
    return _native.lib()


def _backward(lib, saved, sb, B, N, M, gamma, gr, gp, stream, has_p):
    dev = gr.device
    wb = lib.tw_sdtw_workspace_bytes(B, N, M, 4, int(has_p))
    ws = torch.empty(wb, dtype=torch.uint8, device=dev)
    dC = torch.empty(B, N, M, device=dev)
    dQ = torch.empty(B, N, M, device=dev) if has_p else None
    st = lib.tw_sdtw_backward_f32(_p(gr), _p(gp) if has_p else None, B, N, M, gamma,
                                  int(has_p), _p(saved), sb, _p(dC),
                                  _p(dQ) if has_p else None, _p(ws), wb, stream)
    assert st == 0, lib.tw_last_error()
    return dC, (dQ if has_p else torch.zeros(1, device=dev))


@pytest.mark.parametrize("has_p", [True, False], ids=["udtw", "soft_dtw"])
def test_noalloc_forward_matches_workspace_forward(lib, orc, has_p):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, N, M, gamma, band = 300, 150, 170, 0.1, 0.0  # two bands per pair: delay lines in use
    sb = lib.tw_sdtw_saved_bytes(B, N, M, 4, int(has_p))
    wb = lib.tw_sdtw_workspace_bytes(B, N, M, 4, int(has_p))
    assert 0 < wb <= STATIC_BYTES
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    g = torch.Generator().manual_seed(7)
    gr = torch.rand(B, generator=g).to(dev)
    gp = torch.randn(B, generator=g).to(dev)
    for call in range(2):  # two calls in a row, on different inputs
        C = torch.rand(B, N, M, generator=g).to(dev)
        Q = torch.randn(B, N, M, generator=g).to(dev) if has_p else None
        q_ptr = _p(Q) if has_p else None

        saved_ref = torch.empty(sb, dtype=torch.uint8, device=dev)
        ws = torch.empty(wb, dtype=torch.uint8, device=dev)
        r_ref, p_ref = torch.empty(B, device=dev), torch.zeros(B, device=dev)
        st = lib.tw_sdtw_forward_f32(_p(C), q_ptr, B, N, M, gamma, band, _p(r_ref),
                                     _p(p_ref) if has_p else None, _p(saved_ref), sb, _p(ws),
                                     wb, stream)
        assert st == 0, lib.tw_last_error()

        saved = torch.empty(sb, dtype=torch.uint8, device=dev)
        r = torch.full((B,), float("nan"), device=dev)
        p = torch.full((B,), float("nan"), device=dev) if has_p else torch.zeros(B, device=dev)
        st = lib.tw_sdtw_forward_noalloc_f32(_p(C), q_ptr, B, N, M, gamma, band, _p(r),
                                             _p(p) if has_p else None, _p(saved), sb, stream)
        assert st == 0, lib.tw_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(r.cpu().numpy(), r_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(p.cpu().numpy(), p_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)

        # the saved state it wrote drives the backward to the same gradients
        dC, dQ = _backward(lib, saved, sb, B, N, M, gamma, gr, gp, stream, has_p)
        dC_ref, dQ_ref = _backward(lib, saved_ref, sb, B, N, M, gamma, gr, gp, stream, has_p)
        torch.cuda.synchronize()
        np.testing.assert_allclose(dC.cpu().numpy(), dC_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(dQ.cpu().numpy(), dQ_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)

        # and, independently of the other entry point, the float64 CPU oracle
        # (on a few pairs, so it finishes in a second) within the float32 bar
        k = 4
        Cd = C[:k].double().cpu().numpy()
        Qd = Q[:k].double().cpu().numpy() if has_p else None
        o_r, o_p, _, _ = orc.udtw_dp(Cd, Qd, gamma, band)
        np.testing.assert_allclose(r[:k].double().cpu().numpy(), o_r, rtol=1e-5)
        if has_p:
            np.testing.assert_allclose(p[:k].double().cpu().numpy(), o_p, rtol=1e-4, atol=1e-4)


def test_noalloc_forward_rejects_oversized_scratch(lib):
    B, N, M = 4096, 100, 20000
    assert lib.tw_sdtw_workspace_bytes(B, N, M, 4, 0) > STATIC_BYTES
    st = lib.tw_sdtw_forward_noalloc_f32(None, None, B, N, M, 0.1, 0.0, None, None, None, 0,
                                         None)
    assert st == 5  # TW_ERR_WORKSPACE, before any launch
    assert b"static buffer" in lib.tw_last_error()
