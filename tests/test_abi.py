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


def _cpu_calls():
    """One call of every wrapper family and of the public entry points, on CPU tensors."""
    import torch
    bf = torch.bfloat16
    x, w = torch.zeros(4, 64), torch.ones(64)
    u = torch.zeros(1, 8, 32, dtype=bf)
    A = -torch.ones(8, 4)
    Bm = torch.zeros(1, 4, 32, dtype=bf)
    H, W = torch.zeros(16, 64, dtype=bf), torch.zeros(64, 64, dtype=bf)
    lab = torch.zeros(16, dtype=torch.long)
    cs = torch.ones(32, 4)
    q = torch.zeros(1, 2, 32, 8)

    def scan_fn():
        from kernels.mamba_scan import selective_scan_fn
        return selective_scan_fn(u, u, A, Bm, Bm, delta_softplus=True)

    def linear_ce_loss():
        from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
        return ChunkedLinearCrossEntropyLoss()(H, W, lab)

    return {
        "rmsnorm_fwd": lambda: _ak.rmsnorm_fwd(x, w),
        "rmsnorm_bwd": lambda: _ak.rmsnorm_bwd(x, w, x),
        "fused_res_rmsnorm_fwd": lambda: _ak.fused_res_rmsnorm_fwd(x, x, w),
        "softmax_fwd": lambda: _ak.softmax_fwd(x),
        "silu_gate_mul_fwd": lambda: _ak.silu_gate_mul_fwd(x, x),
        "rope_fwd": lambda: _ak.rope_fwd(q, cs, cs),
        "transpose_bt": lambda: _ak.transpose_bt(x.view(1, 4, 64)),
        "ce_rows_fwd": lambda: _ak.ce_rows_fwd(x, lab[:4]),
        "linear_ce_fwdbwd": lambda: _ak.linear_ce_fwdbwd(H, W, lab),
        "tc_gemm": lambda: _ak.tc_gemm(H, W.t()),
        "scan1_fwd": lambda: _ak.scan1_fwd(x.view(1, 4, 64), x.view(1, 4, 64), x.view(1, 4, 64), w, x.view(1, 4, 64)),
        "selective_scan_fwd": lambda: _ak.selective_scan_fwd(u, u, A, Bm, Bm),
        "causal_conv1d_fwd": lambda: _ak.causal_conv1d_fwd(u, torch.ones(8, 4)),
        "selective_scan_fn": scan_fn,
        "ChunkedLinearCrossEntropyLoss": linear_ce_loss,
    }


@pytest.mark.parametrize("name", sorted(_cpu_calls()))
def test_wrappers_refuse_cpu_tensors(name):
    """No CPU or PyTorch fallback anywhere on the product path: every wrapper family and the
    public entry points raise on CPU tensors instead of computing."""
    with pytest.raises((RuntimeError, NotImplementedError)) as e:
        _cpu_calls()[name]()
    assert "CUDA" in str(e.value) or "cuda" in str(e.value), str(e.value)


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
