"""Depthwise causal conv1d CUDA kernels vs the CPU oracle and the golden fixtures
(reference op: autokernel::causal_conv1d, kernels/hip/_torch_ops.py:883-975;
reference parity test: scripts/test_tier2_parity.py:198-240)."""
import pytest
import torch

from conftest import assert_fp32_close, assert_lowp_close, golden
from oracle import hot_path_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(dtype, a, b, what):
    if dtype == torch.float32:
        assert_fp32_close(a, b, what=what)
    else:
        assert_lowp_close(a, b, what=what)


@pytest.mark.parametrize("tag", ["k4", "k3"])
@pytest.mark.parametrize("silu", [False, True])
def test_conv1d_golden_cuda(tag, silu):
    from kernels import _ak
    g = golden("conv1d")
    x, w, b, dy = (torch.from_numpy(g[f"{tag}_{k}"]).to(DEV) for k in ("x", "w", "b", "dy"))
    p = f"{tag}_silu_" if silu else f"{tag}_"
    assert_fp32_close(_ak.causal_conv1d_fwd(x, w, b, silu), g[p + "y"], what="y")
    dx, dw, db = _ak.causal_conv1d_bwd(x, w, b, dy, silu)
    assert_fp32_close(dx, g[p + "dx"], what="dx")
    assert_fp32_close(dw, g[p + "dw"], what="dw")
    assert_fp32_close(db, g[p + "db"], what="db")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,D,T,K", [(2, 64, 2048, 4), (3, 5, 1, 4), (1, 7, 255, 4), (2, 3, 257, 2), (1, 4, 100, 8),
                                     (2, 6, 13, 3), (1, 1, 9, 5), (4, 256, 64, 4)])
@pytest.mark.parametrize("silu", [False, True])
@pytest.mark.parametrize("with_bias", [True, False])
def test_conv1d_fwd_bwd(dtype, B, D, T, K, silu, with_bias):
    from kernels import _ak
    g = torch.Generator().manual_seed(B * 1000 + D * 10 + T + K)
    x = torch.randn(B, D, T, generator=g).to(dtype)
    w = 0.5 * torch.randn(D, K, generator=g)
    b = 0.1 * torch.randn(D, generator=g) if with_bias else None
    dy = torch.randn(B, D, T, generator=g).to(dtype)
    y = _ak.causal_conv1d_fwd(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), silu)
    close(dtype, y, O.causal_conv1d(x, w, b, silu), "y")
    dx, dw, db = _ak.causal_conv1d_bwd(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), dy.to(DEV), silu)
    rdx, rdw, rdb = O.causal_conv1d_grads(x, w, b, dy, silu)
    close(dtype, dx, rdx, "dx")
    tol = 1e-5 if dtype == torch.float32 else 1e-4
    assert_fp32_close(dw, rdw, rtol=tol, what="dw")
    if with_bias:
        assert_fp32_close(db, rdb, rtol=tol, what="db")
    else:
        assert db is None


def test_conv1d_unaligned_and_empty():
    from kernels import _ak
    w = torch.randn(3, 4, device=DEV)
    base = torch.randn(2 * 3 * 64 + 1, device=DEV)
    xs = base[1:].view(2, 3, 64)  # 4-byte offset: scalar path
    assert_fp32_close(_ak.causal_conv1d_fwd(xs, w), O.causal_conv1d(xs.cpu(), w.cpu()), what="unaligned")
    x0 = torch.zeros(0, 3, 64, device=DEV)
    assert _ak.causal_conv1d_fwd(x0, w).shape == (0, 3, 64)
    dx, dw, db = _ak.causal_conv1d_bwd(x0, w, torch.zeros(3, device=DEV), x0)
    assert dx.shape == x0.shape and torch.all(dw == 0) and torch.all(db == 0)


def test_conv1d_rejects_bad_width():
    from kernels import _ak
    x = torch.randn(1, 2, 8, device=DEV)
    with pytest.raises(_ak.AkError):
        _ak.causal_conv1d_fwd(x, torch.randn(2, 9, device=DEV))


def test_conv1d_deterministic():
    from kernels import _ak
    x = torch.randn(8, 128, 1024, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(128, 4, device=DEV)
    b = torch.randn(128, device=DEV)
    dy = torch.randn_like(x)
    r1 = _ak.causal_conv1d_bwd(x, w, b, dy, True)
    r2 = _ak.causal_conv1d_bwd(x, w, b, dy, True)
    for a, c in zip(r1, r2):
        assert torch.equal(a, c)


@pytest.mark.parametrize("under_autocast", [False, True])
def test_conv1d_custom_op_tier2_shape(under_autocast):
    """Shape, dtypes and flow of the reference's tier-2 parity cell (fp16 x, weight, bias)."""
    import kernels.hip._torch_ops  # noqa: F401  (registers torch.ops.autokernel.*)
    torch.manual_seed(42)
    B, D, T, K = 4, 256, 64, 4
    x = torch.randn(B, D, T, device=DEV, dtype=torch.float16)
    w = torch.randn(D, K, device=DEV, dtype=torch.float16)
    b = torch.randn(D, device=DEV, dtype=torch.float16)
    xh, wh, bh = (t.detach().clone().requires_grad_(True) for t in (x, w, b))
    if under_autocast:
        with torch.amp.autocast(device_type="cuda", dtype=torch.float16):
            y = torch.ops.autokernel.causal_conv1d(xh, wh, bh)
    else:
        y = torch.ops.autokernel.causal_conv1d(xh, wh, bh)
    assert y.dtype == torch.float16 and y.shape == x.shape
    y.float().sum().backward()
    assert wh.grad.dtype == torch.float16 and bh.grad.dtype == torch.float16
    dy = torch.ones(B, D, T, dtype=torch.float64)
    rdx, rdw, rdb = O.causal_conv1d_grads(x.cpu(), w.cpu(), b.cpu(), dy)
    assert_lowp_close(y, O.causal_conv1d(x.cpu(), w.cpu(), b.cpu()), what="y")
    assert_lowp_close(xh.grad, rdx, what="dx")
    assert_lowp_close(wh.grad, rdw, rtol=5e-3, what="dw")
    assert_lowp_close(bh.grad, rdb, rtol=5e-3, what="db")


def test_causal_conv1d_fn_shim():
    from causal_conv1d import causal_conv1d_fn
    x = torch.randn(2, 32, 300, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(32, 4, device=DEV, requires_grad=True)
    b = torch.randn(32, device=DEV, requires_grad=True)
    y = causal_conv1d_fn(x, w, b, activation="silu")
    assert_lowp_close(y, O.causal_conv1d(x.detach().cpu(), w.detach().cpu(), b.detach().cpu(), silu=True), what="y")
    dy = torch.randn_like(y)
    y.backward(dy)
    rdx, rdw, rdb = O.causal_conv1d_grads(x.detach().cpu(), w.detach().cpu(), b.detach().cpu(), dy.cpu(), silu=True)
    assert_lowp_close(x.grad, rdx, what="dx")
    assert_fp32_close(w.grad, rdw, rtol=1e-4, what="dw")
    assert_fp32_close(b.grad, rdb, rtol=1e-4, what="db")
