"""The C-ABI library loads and exports every entry point declared in include/*.h.

No compute calls: these run without a GPU.  Argument validation that happens
before any CUDA call is exercised through ctypes.
"""
import ctypes
import re

import pytest

from conftest import REPO
from kernels import _ak


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        names |= set(re.findall(r"AK_API\s+(?:const\s+)?\w+\s*\*?\s*(ak_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "ak_version" in names and "ak_selective_scan_fwd" in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol():
    lib = _ak.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_bindings_cover_every_declared_symbol():
    bound = set(_ak.exported_symbols())
    missing = [n for n in declared_symbols() if n not in bound]
    assert not missing, f"declared but not bound in kernels/_ak.py: {missing}"


def test_version_and_stride():
    assert _ak.lib().ak_version() >= (0 << 16) | (1 << 8)
    assert _ak.state_stride() == 256


def test_shape_validation_reports_error_without_gpu():
    lib = _ak.lib()
    rc = lib.ak_rmsnorm_fwd(None, None, None, None, 4, 0, 1e-6, 0, 0, None)
    assert rc == 3  # AK_ERR_SHAPE
    assert b"bad shape" in lib.ak_last_error()
    rc = lib.ak_selective_scan_fwd(None, None, None, None, None, None, None, None, None, None, None, 1,
                                   2, 4, 16, 65, 1, 1, None)
    assert rc == 3 and b"dstate" in lib.ak_last_error()
    rc = lib.ak_softmax_fwd(None, None, 0, 16, 1, None)  # empty: nothing to do
    assert rc == 0 and lib.ak_last_error() == b""


def test_workspace_queries():
    n = ctypes.c_size_t(0)
    assert _ak.lib().ak_scan1_bwd_workspace_size(2, 300, 40, ctypes.byref(n)) == 0
    assert n.value == (2 * 5 * 40 + 2 * 40) * 4  # 5 chunks of 64 steps + gD partials
    assert _ak.lib().ak_selective_scan_bwd_workspace_size(2, 8, 300, 16, 2, ctypes.byref(n)) == 0
    assert n.value == (2 * 2 * 2 * 16 * 300 + 2 * 8 * 18) * 4


def test_wrappers_refuse_cpu_tensors():
    import torch
    with pytest.raises(RuntimeError, match="CUDA"):
        _ak.rmsnorm_fwd(torch.zeros(2, 8), torch.ones(8))
