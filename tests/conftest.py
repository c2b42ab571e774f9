"""Shared test setup: import paths, the `gpu` marker, tolerance helpers."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "autokernel-halo-strix_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and libak_b200.so")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


# Tolerances (stated once, used everywhere):
#   fp32 paths: max|a - b| <= 1e-5 * max|b|   (norm-relative)
#   bf16/fp16 paths: |a - b| <= 2e-2 + 2e-2 * |b| elementwise, fp32 accumulation
#   (the reference's own bf16 tolerance, kernels/ce_fused.py:47, atol = rtol = 0.02).
FP32_RTOL = 1e-5
LOWP_ATOL = 2e-2
LOWP_RTOL = 2e-2


def to64(t):
    if isinstance(t, np.ndarray):
        return torch.from_numpy(t).double()
    return t.detach().to("cpu", torch.float64)


def assert_fp32_close(actual, expected, rtol=FP32_RTOL, what=""):
    a, b = to64(actual), to64(expected)
    assert a.shape == b.shape, f"{what}: shape {tuple(a.shape)} != {tuple(b.shape)}"
    fin = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), fin), f"{what}: non-finite pattern differs"
    scale = b[fin].abs().max().item() if fin.any() else 0.0
    err = (a[fin] - b[fin]).abs().max().item() if fin.any() else 0.0
    assert err <= rtol * max(scale, 1e-30), f"{what}: max err {err:.3e} > {rtol:g} * {scale:.3e}"


def assert_lowp_close(actual, expected, atol=LOWP_ATOL, rtol=LOWP_RTOL, what=""):
    a, b = to64(actual), to64(expected)
    assert a.shape == b.shape, f"{what}: shape {tuple(a.shape)} != {tuple(b.shape)}"
    fin = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), fin), f"{what}: non-finite pattern differs"
    bad = ((a - b).abs() > atol + rtol * b.abs()) & fin
    if bad.any():
        idx = bad.nonzero()[0].tolist()
        raise AssertionError(f"{what}: {int(bad.sum())} elements out of tolerance, first at {idx}: "
                             f"{a[tuple(idx)].item():.5g} vs {b[tuple(idx)].item():.5g}")
