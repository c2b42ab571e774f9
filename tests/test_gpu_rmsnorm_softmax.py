"""RMSNorm and softmax CUDA kernels vs the CPU oracle and the golden fixtures."""
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


def test_rmsnorm_golden_cuda():
    from kernels.hip import rmsnorm, rmsnorm_backward
    g = golden("rmsnorm")
    x, w, dy = (torch.from_numpy(g[k]).to(DEV) for k in ("x", "w", "dy"))
    assert_fp32_close(rmsnorm.kernel_fn(x, w), g["y"], what="y")
    dx, dw = rmsnorm_backward.kernel_fn(x, w, dy)
    assert dw.dtype == torch.float32
    assert_fp32_close(dx, g["dx_autograd"], what="dx")
    assert_fp32_close(dw, g["dw_autograd"], what="dw")


@pytest.mark.parametrize("dtype,wdtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                          (torch.bfloat16, torch.float32), (torch.float16, torch.float16)])
@pytest.mark.parametrize("M,N", [(8192, 768), (37, 768), (5, 1000), (3, 64), (17, 4096), (2, 8200), (1, 7)])
def test_rmsnorm_fwd_bwd(dtype, wdtype, M, N):
    from kernels import _ak
    g = torch.Generator().manual_seed(M * 31 + N)
    x = torch.randn(M, N, generator=g).to(dtype)
    w = (1 + 0.02 * torch.randn(N, generator=g)).to(wdtype)
    dy = torch.randn(M, N, generator=g).to(dtype)
    y = _ak.rmsnorm_fwd(x.to(DEV), w.to(DEV), 1e-6)
    close(dtype, y, O.rmsnorm_fwd(x, w), "y")
    dx, dw = _ak.rmsnorm_bwd(x.to(DEV), w.to(DEV), dy.to(DEV), 1e-6)
    rdx, rdw = O.rmsnorm_bwd(x, w, dy)
    close(dtype, dx, rdx, "dx")
    assert_fp32_close(dw, rdw, rtol=1e-5 if dtype == torch.float32 else 2e-3, what="dw")


def test_rmsnorm_empty_and_unaligned():
    from kernels import _ak
    x = torch.zeros(0, 768, device=DEV)
    w = torch.ones(768, device=DEV)
    assert _ak.rmsnorm_fwd(x, w).shape == (0, 768)
    dx, dw = _ak.rmsnorm_bwd(x, w, x)
    assert dx.shape == (0, 768) and torch.all(dw == 0)
    base = torch.randn(10 * 768 + 1, device=DEV)
    xs = base[1:].view(10, 768)  # 4-byte offset: not 16-byte aligned
    assert_fp32_close(_ak.rmsnorm_fwd(xs, w), O.rmsnorm_fwd(xs.cpu(), w.cpu()), what="unaligned")


def test_rmsnorm_dw_deterministic():
    from kernels import _ak
    x = torch.randn(8192, 768, device=DEV)
    w = torch.randn(768, device=DEV)
    dy = torch.randn(8192, 768, device=DEV)
    a = _ak.rmsnorm_bwd(x, w, dy)[1]
    b = _ak.rmsnorm_bwd(x, w, dy)[1]
    assert torch.equal(a, b)


def test_rmsnorm_custom_op_autograd():
    import kernels.hip._torch_ops  # noqa: F401
    x = torch.randn(4, 33, 768, device=DEV, requires_grad=True)
    w = torch.randn(768, device=DEV, requires_grad=True)
    y = torch.ops.autokernel.rmsnorm(x.view(-1, 768), w)
    y.sum().backward()
    rdx, rdw = O.rmsnorm_bwd(x.detach().view(-1, 768).cpu(), w.detach().cpu(), torch.ones(132, 768))
    assert_fp32_close(x.grad.view(-1, 768), rdx, what="dx")
    assert_fp32_close(w.grad, rdw, what="dw")
    y2 = torch.ops.autokernel.rmsnorm_eps(x, w, 1e-5)
    assert_fp32_close(y2, O.rmsnorm_fwd(x.detach().cpu(), w.detach().cpu(), 1e-5), what="eps op")


def test_softmax_golden_cuda():
    from kernels.hip import softmax
    g = golden("softmax")
    x = torch.from_numpy(g["x"]).to(DEV).requires_grad_(True)
    y = softmax.kernel_fn(x)
    assert_fp32_close(y, g["y"], what="y")
    y.backward(torch.from_numpy(g["dy"]).to(DEV))
    assert_fp32_close(x.grad, g["dx"], what="dx")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(96 * 16, 2048), (7, 1023), (3, 4097), (2, 50257), (5, 1), (33, 8), (4, 4096)])
def test_softmax_fwd_bwd(dtype, rows, cols):
    from kernels import _ak
    g = torch.Generator().manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=g) / 8).to(dtype)
    if cols == 2048:  # causal mask rows as in attention scores
        L = cols
        r = torch.arange(rows) % L
        x = x.masked_fill(torch.arange(cols)[None, :] > r[:, None], float("-inf"))
    dy = torch.randn(rows, cols, generator=g).to(dtype)
    y = _ak.softmax_fwd(x.to(DEV))
    ry = O.softmax_fwd(x)
    close(dtype, y, ry, "y")
    dx = _ak.softmax_bwd(y, dy.to(DEV))
    close(dtype, dx, O.softmax_bwd(y.cpu(), dy), "dx")


def test_softmax_many_rows_all_written():
    """Every row is computed even beyond 65535 rows (reference grid clamp, softmax.py:293)."""
    from kernels import _ak
    x = torch.randn(70000, 64, device=DEV, dtype=torch.float16)
    y = _ak.softmax_fwd(x)
    s = y.float().sum(-1)
    assert torch.allclose(s, torch.ones_like(s), atol=1e-2)


def test_softmax_all_masked_row_matches_torch():
    from kernels import _ak
    x = torch.full((2, 32), float("-inf"), device=DEV)
    x[1, 3] = 0.0
    y = _ak.softmax_fwd(x)
    ref = torch.softmax(x.cpu().double(), -1)
    assert torch.isnan(y[0]).all() and torch.isnan(ref[0]).all()
    assert_fp32_close(y[1], ref[1], what="row 1")
