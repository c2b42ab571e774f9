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
                                   2, 4, 16, 65, 1, 1, None, None)
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


def test_new_entry_points_validate_before_any_cuda_call():
    """Argument checks of the strided RoPE, the device-scalar scale and the collapsed scan with
    saved states, all before any CUDA call (no GPU here)."""
    lib = _ak.lib()
    fake = ctypes.c_void_p(256)  # never dereferenced: every call below fails validation first
    # ak_rope_strided: mode must be 1, -1 or 0
    rc = lib.ak_rope_strided(fake, fake, fake, fake, 1, 2, 4, 8, 64, 8, 16, 64, 32, 8, 2, 1, None)
    assert rc != 0 and b"mode" in lib.ak_last_error()
    # ... and rotation modes need the tables (copy mode does not)
    rc = lib.ak_rope_strided(fake, fake, None, None, 1, 2, 4, 7, 64, 8, 16, 64, 32, 8, 1, 1, None)
    assert rc != 0 and b"D must be even" in lib.ak_last_error()
    # ak_scale_by_device_scalar: negative size / missing scalar
    assert lib.ak_scale_by_device_scalar(fake, -1, fake, 1, None) != 0
    assert lib.ak_scale_by_device_scalar(fake, 10, None, 1, None) != 0
    assert lib.ak_scale_by_device_scalar(None, 0, None, 1, None) == 0  # empty: nothing to do
    # collapsed scan: carries size and the smaller workspace when they are given
    n = ctypes.c_size_t(0)
    assert lib.ak_scan1_carries_size(2, 300, 40, ctypes.byref(n)) == 0
    assert n.value == 2 * 5 * 40 * 4  # one state per 64-step chunk
    rc = lib.ak_scan1_bwd_ex(fake, fake, fake, fake, fake, fake, ctypes.c_size_t(2 * 40 * 4 - 4), fake, fake, fake,
                             fake, fake, fake, fake, 2, 300, 40, None)
    assert rc != 0 and b"workspace" in lib.ak_last_error()
    rc = lib.ak_scan1_bwd_ex(fake, fake, fake, fake, fake, fake, ctypes.c_size_t(2 * 40 * 4), None, fake, fake,
                             fake, fake, fake, fake, 2, 300, 40, None)  # no carries: needs them in the workspace
    assert rc != 0 and b"workspace" in lib.ak_last_error()
