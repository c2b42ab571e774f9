"""Tiled transpose kernel and the layout ops of the Mamba block (autokernel::transpose_bt,
autokernel::split_transpose) against torch's transpose; bit-exact (pure data movement)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,R,C", [(2, 1024, 1536), (1, 64, 64), (3, 100, 37), (2, 8, 24), (1, 1, 1), (4, 2048, 16)])
def test_transpose_exact(dtype, B, R, C):
    from kernels import _ak
    x = torch.randn(B, R, C, device=DEV).to(dtype)
    assert torch.equal(_ak.transpose_bt(x), x.transpose(1, 2).contiguous())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_transpose_strided_views(dtype):
    from kernels import _ak
    xz = torch.randn(2, 300, 2 * 96, device=DEV).to(dtype)
    for part in (xz[:, :, :96], xz[:, :, 96:]):
        assert torch.equal(_ak.transpose_bt(part), part.transpose(1, 2).contiguous())
    out = torch.zeros(2, 300, 2 * 96, device=DEV, dtype=dtype)
    g = torch.randn(2, 96, 300, device=DEV).to(dtype)
    _ak.transpose_into(out[:, :, 96:], g)
    assert torch.equal(out[:, :, 96:], g.transpose(1, 2))
    assert torch.all(out[:, :, :96] == 0)


def test_layout_ops_autograd():
    import kernels.hip._torch_ops  # noqa: F401
    xz = torch.randn(2, 256, 2 * 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    x, z = torch.ops.autokernel.split_transpose(xz, 64)
    y = torch.ops.autokernel.transpose_bt(x * 2 + z)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr = xz.detach().clone().requires_grad_(True)
    a, b = xr.transpose(1, 2).chunk(2, dim=1)
    (a * 2 + b).transpose(1, 2).backward(gy)
    assert torch.equal(x, xz.detach()[:, :, :64].transpose(1, 2))
    assert torch.equal(xz.grad, xr.grad)


def test_mamba_block_kernel_path_matches_eager():
    import copy

    import kernels.hip._torch_ops  # noqa: F401
    from halo_training.hybrid_lm import HybridConfig, MambaBlock
    torch.manual_seed(0)
    ref = MambaBlock(HybridConfig()).to(DEV)
    fused = copy.deepcopy(ref)
    fused.fused_conv = True
    h = torch.randn(2, 512, 768, device=DEV)
    outs = []
    for m in (ref, fused):
        hi = h.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(hi)
        y.float().square().mean().backward()
        outs.append((y.float(), hi.grad, {n: p.grad for n, p in m.named_parameters()}))
    tol = dict(atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(outs[1][0], outs[0][0], **tol)
    torch.testing.assert_close(outs[1][1], outs[0][1], **tol)
    for n, g in outs[0][2].items():
        torch.testing.assert_close(outs[1][2][n].float(), g.float(), **tol, msg=n)
