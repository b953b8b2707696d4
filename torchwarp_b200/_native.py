"""ctypes binding of libtorchwarp_b200.so (the C ABI in include/torchwarp_b200.h).

The library is built ahead of time (``python -m torchwarp_b200.build``); it is
loaded on first use and a missing or stale build is an error, never a silent
fallback.  Helpers here turn torch tensors into raw pointers and the current
CUDA stream into the ``void* stream`` argument.
"""

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtorchwarp_b200.so"

_c_p = ctypes.c_void_p
_c_i = ctypes.c_int
_c_d = ctypes.c_double
_c_sz = ctypes.c_size_t

# name -> (restype, argtypes); one entry per symbol of include/torchwarp_b200.h
SIGNATURES = {
    "tw_version": (_c_i, []),
    "tw_last_error": (ctypes.c_char_p, []),
    "tw_device_error": (_c_i, []),
    "tw_sdtw_saved_bytes": (_c_sz, [_c_i, _c_i, _c_i, _c_i, _c_i]),
    "tw_sdtw_workspace_bytes": (_c_sz, [_c_i, _c_i, _c_i, _c_i, _c_i]),
    "tw_sdtw_forward_f32": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_d, _c_p, _c_p, _c_p,
                                   _c_sz, _c_p, _c_sz, _c_p]),
    "tw_sdtw_forward_f64": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_d, _c_p, _c_p, _c_p,
                                   _c_sz, _c_p, _c_sz, _c_p]),
    "tw_sdtw_forward_noalloc_f32": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_d, _c_p, _c_p,
                                           _c_p, _c_sz, _c_p]),
    "tw_sdtw_backward_f32": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_i, _c_p, _c_sz, _c_p,
                                    _c_p, _c_p, _c_sz, _c_p]),
    "tw_sdtw_backward_f64": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_i, _c_p, _c_sz, _c_p,
                                    _c_p, _c_p, _c_sz, _c_p]),
    "tw_sdtw_backward_masked_f32": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_sz, _c_p, _c_p,
                                           _c_p, _c_sz, _c_p]),
    "tw_sdtw_backward_masked_f64": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_sz, _c_p, _c_p,
                                           _c_p, _c_sz, _c_p]),
    "tw_sdtw_chunk_flags_bytes": (_c_sz, [_c_i, _c_i, _c_i]),
    "tw_sdtw_backward_masked_flags_f32": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_sz, _c_p,
                                                 _c_p, _c_p, _c_sz, _c_p, _c_sz, _c_p]),
    "tw_sdtw_nonzero_mask_bytes": (_c_sz, [_c_i, _c_i, _c_i]),
    "tw_sdtw_backward_flags_f32": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_i, _c_p, _c_sz,
                                          _c_p, _c_p, _c_p, _c_sz, _c_p, _c_sz, _c_p]),
    "tw_udtw_features_grad_flagged_f32": (_c_i, [_c_p] * 8 + [_c_i] * 4 + [_c_d, _c_d]
                                          + [_c_p] * 5),
    "tw_sdtw_backward_sparse_f32": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_sz, _c_p, _c_p,
                                           _c_p, _c_p, _c_sz, _c_p, _c_sz, _c_p]),
    "tw_sdtw_features_workspace_bytes": (_c_sz, [_c_i, _c_i, _c_i, _c_i]),
    "tw_sdtw_features_backward_f32": (_c_i, [_c_p] * 4 + [_c_i] * 4 + [_c_d, _c_p, _c_sz, _c_p,
                                                                   _c_p, _c_p, _c_sz, _c_p]),
    "tw_sdtw_features_backward_f64": (_c_i, [_c_p] * 4 + [_c_i] * 4 + [_c_d, _c_p, _c_sz, _c_p,
                                                                   _c_p, _c_p, _c_sz, _c_p]),
    "tw_udtw_cost_f32": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_d, _c_d, _c_p,
                                _c_p, _c_p]),
    "tw_udtw_cost_f64": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_d, _c_d, _c_p,
                                _c_p, _c_p]),
    "tw_udtw_features_grad_f32": (_c_i, [_c_p] * 7 + [_c_i] * 4 + [_c_d, _c_d] + [_c_p] * 5),
    "tw_udtw_features_grad_f64": (_c_i, [_c_p] * 7 + [_c_i] * 4 + [_c_d, _c_d] + [_c_p] * 5),
    "tw_sqeuclid_cost_f32": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_p, _c_p, _c_p]),
    "tw_sqeuclid_cost_f64": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_p, _c_p, _c_p]),
    "tw_sqeuclid_grad_f32": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_p, _c_p,
                                    _c_p]),
    "tw_sqeuclid_grad_f64": (_c_i, [_c_p, _c_p, _c_p, _c_p, _c_i, _c_i, _c_i, _c_i, _c_p, _c_p,
                                    _c_p]),
    "tw_sqeuclid_grad_flagged_f32": (_c_i, [_c_p] * 4 + [_c_i] * 4 + [_c_p, _c_p, _c_p]),
    "tw_sqeuclid_grad_sparse_f32": (_c_i, [_c_p] * 5 + [_c_i] * 4 + [_c_p, _c_p, _c_p]),
    "tw_jeanie_forward_f32": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_d, _c_p,
                                     _c_p, _c_p]),
    "tw_jeanie_forward_f64": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_d, _c_p,
                                     _c_p, _c_p]),
    "tw_jeanie_backward_f32": (_c_i, [_c_p, _c_p, _c_p, _c_p] + [_c_i] * 7 + [_c_d, _c_p, _c_p]),
    "tw_jeanie_backward_f64": (_c_i, [_c_p, _c_p, _c_p, _c_p] + [_c_i] * 7 + [_c_d, _c_p, _c_p]),
    "tw_qs_cost_f32": (_c_i, [_c_p, _c_p] + [_c_i] * 5 + [_c_p, _c_p]),
    "tw_qs_cost_f64": (_c_i, [_c_p, _c_p] + [_c_i] * 5 + [_c_p, _c_p]),
    "tw_qs_cost_grad_f32": (_c_i, [_c_p] * 4 + [_c_i] * 5 + [_c_p, _c_p, _c_p]),
    "tw_qs_cost_grad_f64": (_c_i, [_c_p] * 4 + [_c_i] * 5 + [_c_p, _c_p, _c_p]),
    "tw_qs_rbf_cost_f32": (_c_i, [_c_p, _c_p] + [_c_i] * 4 + [_c_d, _c_p, _c_p]),
    "tw_qs_rbf_cost_f64": (_c_i, [_c_p, _c_p] + [_c_i] * 4 + [_c_d, _c_p, _c_p]),
    "tw_qs_rbf_cost_grad_f32": (_c_i, [_c_p] * 3 + [_c_i] * 4 + [_c_d] + [_c_p] * 3),
    "tw_qs_rbf_cost_grad_f64": (_c_i, [_c_p] * 3 + [_c_i] * 4 + [_c_d] + [_c_p] * 3),
    "tw_fvm_softmin_f32": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_p]),
    "tw_fvm_softmin_f64": (_c_i, [_c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_p]),
    "tw_fvm_softmin_backward_f32": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_p]),
    "tw_fvm_softmin_backward_f64": (_c_i, [_c_p, _c_p, _c_i, _c_i, _c_i, _c_d, _c_p, _c_p]),
    "tw_jeanie_fused_supported": (_c_i, [_c_i] * 6),
    "tw_jeanie_fused_saved_bytes": (_c_sz, [_c_i] * 6),
    "tw_jeanie_fused_forward_f32": (_c_i, [_c_p] * 3 + [_c_i] * 10 + [_c_d, _c_p, _c_p, _c_p, _c_sz,
                                                                  _c_p]),
    "tw_jeanie_fused_backward_f32": (_c_i, [_c_p] * 5 + [_c_i] * 10 + [_c_d, _c_p, _c_sz, _c_p,
                                                                   _c_p, _c_p, _c_p]),
    "tw_optimal_path_f64": (_c_i, [_c_p] + [_c_i] * 6 + [_c_p] * 5),
}

_LIB = None


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def lib():
    """Load (once) and return the CDLL with every signature declared."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                "torchwarp_b200: native library {} is missing; build it with "
                "`python -m torchwarp_b200.build` (CUDA 12.9+, sm_100a)".format(LIB_PATH))
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status, what):
    if status != 0:
        msg = lib().tw_last_error().decode(errors="replace")
        raise NativeError("{} failed (status {}): {}".format(what, status, msg))


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def suffix(dtype):
    if dtype == torch.float32:
        return "f32"
    if dtype == torch.float64:
        return "f64"
    raise TypeError("torchwarp_b200 kernels take float32 or float64, got {}".format(dtype))


def require_cuda(*tensors):
    """The native path is the only path: CPU tensors are rejected loudly."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "torchwarp_b200 runs only on CUDA tensors (B200, sm_100a); got a tensor on {}. "
                "There is no CPU fallback.".format(t.device))


# ------------------------------------------------------------ launch timing
#
# bench.py measures each native launch with CUDA events recorded on the
# launching stream.  The recorder is off by default and adds nothing to a
# call when it is off.

_RECORDER = None


class LaunchTimer:
    """Context manager collecting (name, start_event, end_event) per C-ABI call."""

    def __init__(self):
        self.events = []

    def __enter__(self):
        global _RECORDER
        _RECORDER = self
        return self

    def __exit__(self, *exc):
        global _RECORDER
        _RECORDER = None
        return False

    def totals(self):
        """{name: (launches, total_ms)} after a torch.cuda.synchronize()."""
        out = {}
        for name, a, b in self.events:
            n, ms = out.get(name, (0, 0.0))
            out[name] = (n + 1, ms + a.elapsed_time(b))
        return out


def call(name, fn, *args):
    """Invoke a C-ABI function, bracketing it with CUDA events when timing."""
    rec = _RECORDER
    if rec is None:
        return fn(*args)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    status = fn(*args)
    b.record()
    rec.events.append((name, a, b))
    return status
