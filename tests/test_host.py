"""Host-side checks that need no GPU: the C ABI library, the public API surface,
argument validation and the no-CPU-fallback policy.

The validation cases restate the reference's own host tests
(hibana2077/torchwarp tests/test_udtw.py:239-250, tests/test_jeanie.py:335-353,
tests/test_public_api.py:20-35, 225-251): same exceptions on the same inputs.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

import torchwarp_b200 as tw
import torchwarp_b200.functional as TF
from torchwarp_b200 import FVM, JEANIE, UDTW, _native

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "torchwarp_b200.h"


def _header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tw_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    declared = _header_functions()
    assert len(declared) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tw_[a-z0-9_]+)", out))
    missing = [n for n in declared if n not in exported]
    assert not missing, missing
    for name in declared:
        assert hasattr(lib, name)
        assert name in _native.SIGNATURES, name


def _header_param_types():
    """{function: [parameter type per parameter]} of the header's declarations."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(tw_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in m.group(2).split(",") if p.strip() not in ("", "void")]
        out[m.group(1)] = [re.sub(r"\s*\b[A-Za-z_][A-Za-z0-9_]*$", "", p) for p in params]
    return out


def _ctype_of(decl):
    if "*" in decl:
        return ctypes.c_void_p
    if "size_t" in decl:
        return ctypes.c_size_t
    if "double" in decl:
        return ctypes.c_double
    return ctypes.c_int


def test_ctypes_signatures_match_header():
    """Every ctypes binding has the header's parameter count and kinds
    (pointer, size_t, double, int): a mismatch would pass garbage through the
    C ABI on the GPU box."""
    decls = _header_param_types()
    assert len(decls) == len(_header_functions())
    for name, params in decls.items():
        _, argtypes = _native.SIGNATURES[name]
        assert len(argtypes) == len(params), (name, len(argtypes), len(params))
        for k, (decl, got) in enumerate(zip(params, argtypes)):
            assert got is _ctype_of(decl), (name, k, decl, got)


def test_library_host_calls_without_gpu():
    lib = _native.lib()
    assert lib.tw_version() >= 100
    # argument errors are reported through the status and tw_last_error, no launch
    st = lib.tw_udtw_cost_f32(None, None, None, None, 1, 0, 4, 3, 0.0, 1e-8, None, None, None)
    assert st == 1
    assert b"invalid" in lib.tw_last_error()
    st = lib.tw_jeanie_forward_f64(None, 1, 0, 1, 4, 4, 0, 0, 0.1, None, None, None)
    assert st == 1
    st = lib.tw_optimal_path_f64(None, 1, 2, 3, 3, 0, 5, None, None, None, None, None)
    assert st == 1


def test_exports_match_reference_api():
    for name in ("UDTW", "SoftDTW", "JEANIE", "FVM", "euclidean_cost", "squared_euclidean_cost",
                 "rbf_cost", "functional", "paths"):
        assert hasattr(tw, name), name
    for name in ("udtw", "udtw_from_cost", "pairwise_matrices", "UDTWOutput", "soft_dtw",
                 "soft_dtw_from_cost", "jeanie", "jeanie_from_cost", "fvm", "fvm_from_cost",
                 "softmin", "softmin_weights", "euclidean_cost", "squared_euclidean_cost",
                 "rbf_cost"):
        assert hasattr(TF, name), name
    assert tw.__version__
    with pytest.raises(TypeError):
        UDTW(use_cuda=False)
    with pytest.raises(TypeError):
        tw.SoftDTW(use_cuda=False)


def _udtw_inputs(B=2, N=4, M=5):
    g = torch.Generator().manual_seed(0)
    return (torch.rand(B, N, 5, generator=g), torch.rand(B, M, 5, generator=g),
            0.5 + torch.rand(B, N, 1, generator=g), 0.5 + torch.rand(B, M, 1, generator=g))


def test_udtw_validation():
    X, Y, SX, SY = _udtw_inputs()
    with pytest.raises(ValueError):
        UDTW(gamma=0.0)
    with pytest.raises(ValueError):
        UDTW(gamma=0.1, beta=-1.0)
    with pytest.raises(ValueError):
        UDTW(gamma=0.1)(X[0], Y, SX, SY)
    with pytest.raises(ValueError):
        UDTW(gamma=0.1)(X[0], Y[0], SX[0], SY[0])
    with pytest.raises(ValueError):
        UDTW(gamma=0.1, backend="nope")
    with pytest.raises(ValueError):
        UDTW(gamma=0.1, method="nope")
    with pytest.raises(TypeError):
        TF.udtw(X, Y, SX, SY, 0.1, 1.0)
    with pytest.raises(TypeError):
        TF.udtw_from_cost(torch.rand(1, 3, 4), torch.rand(1, 3, 4), 0.1)
    with pytest.raises(ValueError):
        TF.udtw_from_cost(torch.rand(3, 4), torch.rand(3, 4))


def test_jeanie_validation():
    with pytest.raises(ValueError):
        TF.jeanie_from_cost(torch.rand(4, 5), gamma=0.1)
    with pytest.raises(ValueError):
        TF.jeanie_from_cost(torch.rand(2, 4, 5), gamma=0.1)
    with pytest.raises(ValueError):
        TF.jeanie_from_cost(torch.rand(1, 2, 4, 5), gamma=0.0)
    with pytest.raises(ValueError):
        TF.jeanie_from_cost(torch.rand(1, 2, 4, 5), gamma=0.1, max_shift=-1)
    with pytest.raises(ValueError):
        TF.jeanie(torch.rand(2, 4, 3), torch.rand(5, 3))
    with pytest.raises(TypeError):
        TF.soft_dtw_from_cost(torch.ones(1, 3, 3, dtype=torch.int64))
    with pytest.raises(ValueError):
        TF.soft_dtw_from_cost(torch.rand(3, 3))
    with pytest.raises(ValueError):
        TF.fvm_from_cost(torch.rand(4, 5, 6))
    with pytest.raises(TypeError):
        TF.jeanie_from_cost(torch.rand(1, 2, 4, 5), 0.1)
    with pytest.raises(TypeError):
        TF.fvm_from_cost(torch.rand(1, 2, 3, 4), 0.1)
    with pytest.raises(TypeError):
        TF.soft_dtw_from_cost(torch.rand(1, 3, 4), 0.1)
    with pytest.raises(ValueError):
        JEANIE(gamma=0.1, max_shift=(1, 1))(torch.rand(2, 3, 4, 5), torch.rand(2, 6, 5))
    with pytest.raises(ValueError):
        TF.jeanie(torch.rand(2, 3, 2, 4, 5), torch.rand(2, 6, 5), max_shift=(1, 1, 1))
    with pytest.raises(ValueError):
        FVM(gamma=0.1, metric="cosine")
    assert "max_shift=(1, 1)" in repr(JEANIE(gamma=0.1, max_shift=(1, 1)))


def test_softmin_is_torch_level():
    v = torch.randn(3, 4, dtype=torch.float64)
    torch.testing.assert_close(TF.softmin_weights(v, 0.5, dim=1), torch.softmax(-v / 0.5, dim=1))
    torch.testing.assert_close(TF.softmin(v, 0.5, dim=1), -0.5 * torch.logsumexp(-v / 0.5, dim=1))


@pytest.mark.parametrize("call", [
    lambda: TF.soft_dtw_from_cost(torch.rand(1, 3, 4), gamma=0.1),
    lambda: TF.soft_dtw(torch.rand(1, 3, 2), torch.rand(1, 4, 2), gamma=0.1),
    lambda: TF.udtw(*_udtw_inputs(), gamma=0.1),
    lambda: TF.jeanie_from_cost(torch.rand(1, 2, 3, 4), gamma=0.1),
    lambda: TF.jeanie(torch.rand(1, 2, 3, 4), torch.rand(1, 5, 4), gamma=0.1),
    lambda: TF.fvm_from_cost(torch.rand(1, 2, 3, 4), gamma=0.1),
    lambda: tw.euclidean_cost(torch.rand(2, 3, 4), torch.rand(2, 5, 4)),
    lambda: tw.rbf_cost(torch.rand(2, 3, 4), torch.rand(2, 5, 4)),
    lambda: TF.fvm(torch.rand(1, 2, 3, 4), torch.rand(1, 2, 5, 4), gamma=0.1, metric="rbf"),
    lambda: torch.func.jvp(lambda c: TF.soft_dtw_from_cost(c, gamma=0.1),
                           (torch.rand(1, 3, 4),), (torch.rand(1, 3, 4),)),
    lambda: tw.paths.optimal_path(torch.rand(1, 3, 4)),
])
def test_no_cpu_fallback(call):
    """The native kernels are the only implementation: CPU tensors fail loudly."""
    with pytest.raises(RuntimeError, match="CUDA"):
        call()


def test_torch_backend_refused():
    with pytest.raises(RuntimeError, match="no PyTorch"):
        TF.soft_dtw_from_cost(torch.rand(1, 3, 4), gamma=0.1, backend="torch")


def test_oracle_is_not_imported_by_the_package():
    import sys
    for name in list(sys.modules):
        if name.startswith("torchwarp_b200"):
            mod = sys.modules[name]
            src = getattr(mod, "__file__", None)
            if src and src.endswith(".py"):
                assert "import oracle" not in Path(src).read_text(), name
    for p in (ROOT / "torchwarp_b200").rglob("*.py"):
        assert "oracle" not in p.read_text().replace("no CPU", ""), p


def test_plan_is_pure_host_logic():
    # sizes of the saved stream / workspace are defined without touching a GPU
    lib = _native.lib()
    sb = lib.tw_sdtw_saved_bytes(4096, 1024, 1024, 4, 0)
    wb = lib.tw_sdtw_workspace_bytes(4096, 1024, 1024, 4, 0)
    assert sb >= 4096 * 1024 * 1024 * 4
    assert 0 < wb < sb
    assert ctypes.sizeof(ctypes.c_void_p) == 8
