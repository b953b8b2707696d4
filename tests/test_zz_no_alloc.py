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


def _backward(lib, saved, sb, B, N, M, gamma, gr, gp, stream):
    dev = gr.device
    wb = lib.tw_sdtw_workspace_bytes(B, N, M, 4, 1)
    ws = torch.empty(wb, dtype=torch.uint8, device=dev)
    dC = torch.empty(B, N, M, device=dev)
    dQ = torch.empty(B, N, M, device=dev)
    st = lib.tw_sdtw_backward_f32(_p(gr), _p(gp), B, N, M, gamma, 1, _p(saved), sb, _p(dC),
                                  _p(dQ), _p(ws), wb, stream)
    assert st == 0, lib.tw_last_error()
    return dC, dQ


def test_noalloc_forward_matches_workspace_forward(lib):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, N, M, gamma, band = 300, 150, 170, 0.1, 0.0  # two bands per pair: delay lines in use
    sb = lib.tw_sdtw_saved_bytes(B, N, M, 4, 1)
    wb = lib.tw_sdtw_workspace_bytes(B, N, M, 4, 1)
    assert 0 < wb <= STATIC_BYTES
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    g = torch.Generator().manual_seed(7)
    gr = torch.rand(B, generator=g).to(dev)
    gp = torch.randn(B, generator=g).to(dev)
    for call in range(2):  # two calls in a row, on different inputs
        C = torch.rand(B, N, M, generator=g).to(dev)
        Q = torch.randn(B, N, M, generator=g).to(dev)

        saved_ref = torch.empty(sb, dtype=torch.uint8, device=dev)
        ws = torch.empty(wb, dtype=torch.uint8, device=dev)
        r_ref, p_ref = torch.empty(B, device=dev), torch.empty(B, device=dev)
        st = lib.tw_sdtw_forward_f32(_p(C), _p(Q), B, N, M, gamma, band, _p(r_ref), _p(p_ref),
                                     _p(saved_ref), sb, _p(ws), wb, stream)
        assert st == 0, lib.tw_last_error()

        saved = torch.empty(sb, dtype=torch.uint8, device=dev)
        r = torch.full((B,), float("nan"), device=dev)
        p = torch.full((B,), float("nan"), device=dev)
        st = lib.tw_sdtw_forward_noalloc_f32(_p(C), _p(Q), B, N, M, gamma, band, _p(r), _p(p),
                                             _p(saved), sb, stream)
        assert st == 0, lib.tw_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(r.cpu().numpy(), r_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(p.cpu().numpy(), p_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)

        # the saved state it wrote drives the backward to the same gradients
        dC, dQ = _backward(lib, saved, sb, B, N, M, gamma, gr, gp, stream)
        dC_ref, dQ_ref = _backward(lib, saved_ref, sb, B, N, M, gamma, gr, gp, stream)
        torch.cuda.synchronize()
        np.testing.assert_allclose(dC.cpu().numpy(), dC_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(dQ.cpu().numpy(), dQ_ref.cpu().numpy(), rtol=RTOL, atol=ATOL)


def test_noalloc_forward_rejects_oversized_scratch(lib):
    B, N, M = 4096, 100, 20000
    assert lib.tw_sdtw_workspace_bytes(B, N, M, 4, 0) > STATIC_BYTES
    st = lib.tw_sdtw_forward_noalloc_f32(None, None, B, N, M, 0.1, 0.0, None, None, None, 0,
                                         None)
    assert st == 5  # TW_ERR_WORKSPACE, before any launch
    assert b"static buffer" in lib.tw_last_error()
