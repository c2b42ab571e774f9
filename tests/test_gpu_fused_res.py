"""Fused residual add + RMSNorm CUDA kernels vs the CPU oracle and the golden
fixtures (reference: kernels/hip/fused_residual_add_rmsnorm.py,
fused_residual_rmsnorm_backward.py, autokernel::fused_res_rmsnorm in
kernels/hip/_torch_ops.py:238-303; parity test scripts/test_tier2_parity.py:140-190)."""
import pytest
import torch
import torch.nn as nn

from conftest import assert_fp32_close, assert_lowp_close, golden
from oracle import hot_path_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(dtype, a, b, what):
    if dtype == torch.float32:
        assert_fp32_close(a, b, what=what)
    else:
        assert_lowp_close(a, b, what=what)


def test_fused_res_golden_cuda():
    from kernels.hip import fused_residual_add_rmsnorm as fra
    from kernels.hip import fused_residual_rmsnorm_backward as frb
    g = golden("fused_res")
    x, r, w, gh, gn = (torch.from_numpy(g[k]).to(DEV) for k in ("x", "residual", "w", "grad_hidden", "grad_normed"))
    h, y = fra.kernel_fn_dual(x, r, w)
    assert_fp32_close(h, g["hidden"], what="hidden")
    assert_fp32_close(y, g["normed"], what="normed")
    assert_fp32_close(fra.kernel_fn(x, r, w), g["single"], what="single")
    dx, dres, dw = frb.kernel_fn(h, w, gh, gn)
    assert_fp32_close(dx, g["dx_autograd"], what="dx")
    assert_fp32_close(dres, g["dres_autograd"], what="dres")
    assert_fp32_close(dw, g["dw_autograd"], what="dw")


@pytest.mark.parametrize("dtype,wdtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                          (torch.bfloat16, torch.float32), (torch.float16, torch.float16)])
@pytest.mark.parametrize("M,N", [(8192, 768), (37, 768), (5, 1000), (3, 64), (17, 4096), (2, 8200), (1, 7)])
def test_fused_res_fwd_bwd(dtype, wdtype, M, N):
    from kernels import _ak
    g = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn(M, N, generator=g).to(dtype)
    r = torch.randn(M, N, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(N, generator=g)).to(wdtype)
    gh = torch.randn(M, N, generator=g).to(dtype)
    gn = torch.randn(M, N, generator=g).to(dtype)
    h, y = _ak.fused_res_rmsnorm_fwd(x.to(DEV), r.to(DEV), w.to(DEV), 1e-6)
    rh, ry = O.fused_res_rmsnorm(x, r, w, round_to=None if dtype == torch.float32 else dtype)
    close(dtype, h, rh, "hidden")
    if dtype != torch.float32:  # the rounded sum is bit-exact: same fp32 add, one rounding
        assert torch.equal(h.cpu(), rh.to(dtype))
    close(dtype, y, ry, "normed")
    dx, dw = _ak.fused_res_rmsnorm_bwd(h, w.to(DEV), gh.to(DEV), gn.to(DEV), 1e-6)
    rdx, rdw = O.fused_res_rmsnorm_bwd(h.cpu(), w, gh, gn)
    close(dtype, dx, rdx, "dx")
    assert_fp32_close(dw, rdw, rtol=1e-5 if dtype == torch.float32 else 2e-3, what="dw")


def test_fused_res_without_grad_hidden_matches_rmsnorm_bwd():
    from kernels import _ak
    h = torch.randn(300, 768, device=DEV)
    w = torch.randn(768, device=DEV)
    gn = torch.randn(300, 768, device=DEV)
    dx, dw = _ak.fused_res_rmsnorm_bwd(h, w, None, gn)
    rx, rw = _ak.rmsnorm_bwd(h, w, gn)
    assert torch.equal(dx, rx) and torch.equal(dw, rw)


def test_fused_res_unaligned_and_empty():
    from kernels import _ak
    w = torch.ones(768, device=DEV)
    base = torch.randn(2, 10 * 768 + 1, device=DEV)
    xs, rs = base[0, 1:].view(10, 768), base[1, 1:].view(10, 768)  # 4-byte offsets: block path
    h, y = _ak.fused_res_rmsnorm_fwd(xs, rs, w)
    rh, ry = O.fused_res_rmsnorm(xs.cpu(), rs.cpu(), w.cpu())
    assert_fp32_close(h, rh, what="hidden")
    assert_fp32_close(y, ry, what="normed")
    x0 = torch.zeros(0, 768, device=DEV)
    h0, y0 = _ak.fused_res_rmsnorm_fwd(x0, x0, w)
    assert h0.shape == (0, 768) and y0.shape == (0, 768)


@pytest.mark.parametrize("under_autocast", [False, True])
def test_fused_res_custom_op_tier2_cell(under_autocast):
    """The reference's tier-2 parity cell: fp16 (16*512, 768), both outputs summed."""
    import kernels.hip._torch_ops  # noqa: F401
    torch.manual_seed(42)
    M, N = 16 * 512, 768
    x = torch.randn(M, N, device=DEV, dtype=torch.float16)
    r = torch.randn(M, N, device=DEV, dtype=torch.float16)
    w = torch.randn(N, device=DEV, dtype=torch.float16)
    xh, rh, wh = (t.detach().clone().requires_grad_(True) for t in (x, r, w))
    if under_autocast:
        with torch.amp.autocast(device_type="cuda", dtype=torch.float16):
            hid, nrm = torch.ops.autokernel.fused_res_rmsnorm(xh, rh, wh)
    else:
        hid, nrm = torch.ops.autokernel.fused_res_rmsnorm(xh, rh, wh)
    assert hid.dtype == torch.float16 and nrm.dtype == torch.float16
    (hid.float().sum() + nrm.float().sum()).backward()
    oh, oy = O.fused_res_rmsnorm(x.cpu(), r.cpu(), w.cpu(), round_to=torch.float16)
    assert_lowp_close(hid, oh, what="hidden")
    assert_lowp_close(nrm, oy, what="normed")
    ones = torch.ones(M, N, dtype=torch.float64)
    rdx, rdw = O.fused_res_rmsnorm_bwd(oh, w.cpu(), ones, ones)
    assert_lowp_close(xh.grad, rdx, what="dx")
    assert torch.equal(xh.grad, rh.grad)
    assert_lowp_close(wh.grad, rdw, rtol=1e-2, what="dw")


class _Block(nn.Module):
    def __init__(self, d=256):
        super().__init__()
        self.attention_norm = nn.RMSNorm(d, eps=1e-6)
        self.attention = nn.Linear(d, d)
        self.ffn_norm = nn.RMSNorm(d, eps=1e-5)
        self.feed_forward = nn.Sequential(nn.Linear(d, 2 * d), nn.SiLU(), nn.Linear(2 * d, d))

    def forward(self, x):
        h = x + self.attention(self.attention_norm(x))
        return h + self.feed_forward(self.ffn_norm(h))


@pytest.mark.parametrize("autocast", [False, True])
def test_fused_residual_pattern_matches_eager(autocast):
    import copy

    import autokernel
    torch.manual_seed(0)
    ref = nn.Sequential(_Block()).to(DEV)  # the root module itself is never replaced
    opt = autokernel.optimize(copy.deepcopy(ref), training=True)
    assert autokernel.report(opt)["patterns"]["fused_residual_rmsnorm"]["modules_replaced"] == 1
    x = torch.randn(4, 64, 256, device=DEV)
    outs = []
    for m in (ref, opt):
        xi = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            y = m(xi)
        y.float().square().mean().backward()
        outs.append((y.float(), xi.grad, {n: p.grad for n, p in m.named_parameters()}))
    tol = dict(atol=2e-2, rtol=2e-2) if autocast else dict(atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(outs[1][0], outs[0][0], **tol)
    torch.testing.assert_close(outs[1][1], outs[0][1], **tol)
    assert set(outs[1][2]) == set(outs[0][2])
    for n, g in outs[0][2].items():
        torch.testing.assert_close(outs[1][2][n].float(), g.float(), **tol, msg=n)


@pytest.mark.parametrize("lo", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N", [(4096, 768), (37, 1000), (3, 64)])
def test_mixed_precision_rmsnorm_equals_fp32_kernel_rounded(lo, M, N):
    """fp32 residual stream, 16-bit edges: the mixed kernels do the fp32 kernels' arithmetic and
    round once at the 16-bit outputs, so they match them exactly."""
    from kernels import _ak
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, N, generator=g).to(DEV)
    w = (1 + 0.1 * torch.randn(N, generator=g)).to(DEV)
    a = torch.randn(M, N, generator=g).to(lo).to(DEV)
    gn = torch.randn(M, N, generator=g).to(lo).to(DEV)
    gh = torch.randn(M, N, generator=g).to(DEV)
    # plain norm
    y = _ak.rmsnorm_fwd_mixed(x, w, 1e-6, lo)
    assert y.dtype == lo and torch.equal(y, _ak.rmsnorm_fwd(x, w, 1e-6).to(lo))
    dx, _, dw = _ak.rmsnorm_bwd_mixed(x, w, gn, 1e-6)
    rdx, rdw = _ak.rmsnorm_bwd(x, w, gn.float(), 1e-6)
    assert torch.equal(dx, rdx) and torch.equal(dw, rdw)
    # fused residual
    h, n = _ak.fused_res_rmsnorm_fwd_mixed(a, x, w, 1e-6)
    rh, rn = _ak.fused_res_rmsnorm_fwd(a.float(), x, w, 1e-6)
    assert h.dtype == torch.float32 and n.dtype == lo
    assert torch.equal(h, rh) and torch.equal(n, rn.to(lo))
    dres, dlo, dw2 = _ak.rmsnorm_bwd_mixed(h, w, gn, 1e-6, grad_hidden=gh, want_lo=True)
    rdx2, rdw2 = _ak.fused_res_rmsnorm_bwd(rh, w, gh, gn.float(), 1e-6)
    assert torch.equal(dres, rdx2) and torch.equal(dlo, rdx2.to(lo)) and torch.equal(dw2, rdw2)


def test_mixed_precision_ops_autograd():
    import kernels.hip._torch_ops  # noqa: F401
    x = torch.randn(256, 768, device=DEV, requires_grad=True)
    a = torch.randn(256, 768, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.ones(768, device=DEV, requires_grad=True)
    h, n = torch.ops.autokernel.fused_res_rmsnorm_mixed(a, x, w, 1e-6)
    y = torch.ops.autokernel.rmsnorm_mixed(h, w, 1e-6, torch.bfloat16)
    (h.sum() + n.float().square().sum() + y.float().sum()).backward()
    xr, ar, wr = (t.detach().clone().float().requires_grad_(True) for t in (x, a, w))
    hr = ar + xr
    def nrm(t):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    (hr.sum() + nrm(hr).square().sum() + nrm(hr).sum()).backward()
    torch.testing.assert_close(x.grad, xr.grad, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(a.grad.float(), ar.grad, atol=5e-2, rtol=2e-2)
    assert a.grad.dtype == torch.bfloat16 and x.grad.dtype == torch.float32
    torch.testing.assert_close(w.grad, wr.grad, atol=5e-1, rtol=2e-2)
