"""SiLU gate multiply CUDA kernels vs the CPU oracle and the golden fixtures
(reference: kernels/hip/silu_gate_mul.py, silu_gate_mul_backward.py,
autokernel::silu_gate_mul in kernels/hip/_torch_ops.py:181-231; parity test
scripts/test_tier2_parity.py:52-87)."""
import copy

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from conftest import assert_fp32_close, assert_lowp_close, golden
from oracle import hot_path_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(dtype, a, b, what):
    if dtype == torch.float32:
        assert_fp32_close(a, b, what=what)
    else:
        assert_lowp_close(a, b, what=what)


def test_silu_gate_golden_cuda():
    from kernels.hip import silu_gate_mul, silu_gate_mul_backward
    g = golden("silu_gate")
    gate, up, dy = (torch.from_numpy(g[k]).to(DEV) for k in ("gate", "up", "dy"))
    assert_fp32_close(silu_gate_mul.kernel_fn(gate, up), g["y"], what="y")
    dg, du = silu_gate_mul_backward.kernel_fn(gate, up, dy)
    assert_fp32_close(dg, g["dgate_autograd"], what="dgate")
    assert_fp32_close(du, g["dup_autograd"], what="dup")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(8192, 2048), (37, 1000), (5, 7), (1, 8), (3, 4, 520), (1, 1)])
def test_silu_gate_fwd_bwd(dtype, shape):
    from kernels import _ak
    g = torch.Generator().manual_seed(sum(shape))
    gate = (3 * torch.randn(*shape, generator=g)).to(dtype)
    up = torch.randn(*shape, generator=g).to(dtype)
    dy = torch.randn(*shape, generator=g).to(dtype)
    close(dtype, _ak.silu_gate_mul_fwd(gate.to(DEV), up.to(DEV)), O.silu_gate_mul(gate, up), "y")
    dg, du = _ak.silu_gate_mul_bwd(gate.to(DEV), up.to(DEV), dy.to(DEV))
    rdg, rdu = O.silu_gate_mul_bwd(gate, up, dy)
    close(dtype, dg, rdg, "dgate")
    close(dtype, du, rdu, "dup")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H", [2048, 1000, 3])
def test_silu_gate_packed_halves(dtype, H):
    """gate / up as the halves of one (rows, 2H) tensor, and the packed gradient."""
    from kernels import _ak
    gu = torch.randn(3, 50, 2 * H, device=DEV).to(dtype)
    dy = torch.randn(3, 50, H, device=DEV).to(dtype)
    gate, up = gu[..., :H], gu[..., H:]
    y = _ak.silu_gate_mul_fwd(gate, up)
    close(dtype, y, O.silu_gate_mul(gate.cpu(), up.cpu()), "y")
    packed = torch.empty_like(gu)
    dg, du = _ak.silu_gate_mul_bwd(gate, up, dy, packed_out=packed)
    rdg, rdu = O.silu_gate_mul_bwd(gate.cpu(), up.cpu(), dy.cpu())
    close(dtype, packed[..., :H], rdg, "packed dgate")
    close(dtype, packed[..., H:], rdu, "packed dup")
    assert dg.data_ptr() == packed.data_ptr()


def test_silu_gate_extreme_inputs():
    from kernels import _ak
    gate = torch.tensor([[-1e4, -100.0, -20.0, 0.0, 20.0, 100.0, 1e4, -0.0]], device=DEV)
    up = torch.ones_like(gate)
    y = _ak.silu_gate_mul_fwd(gate, up)
    assert torch.isfinite(y).all()
    assert_fp32_close(y, O.silu_gate_mul(gate.cpu(), up.cpu()), what="y")
    dg, du = _ak.silu_gate_mul_bwd(gate, up, torch.ones_like(gate))
    rdg, rdu = O.silu_gate_mul_bwd(gate.cpu(), up.cpu(), torch.ones(1, 8))
    assert_fp32_close(dg, rdg, what="dgate")
    assert_fp32_close(du, rdu, what="dup")


@pytest.mark.parametrize("under_autocast", [False, True])
def test_silu_gate_custom_op_tier2_cell(under_autocast):
    import kernels.hip._torch_ops  # noqa: F401
    torch.manual_seed(42)
    shape = (16 * 512, 2048)
    gate = torch.randn(shape, device=DEV, dtype=torch.float16)
    up = torch.randn(shape, device=DEV, dtype=torch.float16)
    gh, uh = gate.clone().requires_grad_(True), up.clone().requires_grad_(True)
    with torch.amp.autocast(device_type="cuda", dtype=torch.float16, enabled=under_autocast):
        y = torch.ops.autokernel.silu_gate_mul(gh, uh)
    assert y.dtype == torch.float16
    y.float().sum().backward()
    assert_lowp_close(y, O.silu_gate_mul(gate.cpu(), up.cpu()), what="y")
    rdg, rdu = O.silu_gate_mul_bwd(gate.cpu(), up.cpu(), torch.ones(shape, dtype=torch.float64))
    assert_lowp_close(gh.grad, rdg, what="dgate")
    assert_lowp_close(uh.grad, rdu, what="dup")


class _SwiGLU(nn.Module):
    def __init__(self, d=256, h=512):
        super().__init__()
        self.w1, self.w2, self.w3 = nn.Linear(d, h, bias=False), nn.Linear(h, d, bias=False), nn.Linear(d, h)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class _Packed(nn.Module):
    def __init__(self, d=256, h=512):
        super().__init__()
        self.w_gate_up, self.w_down = nn.Linear(d, 2 * h), nn.Linear(h, d)

    def forward(self, x):
        g, u = self.w_gate_up(x).chunk(2, dim=-1)
        return self.w_down(F.silu(g) * u)


@pytest.mark.parametrize("cls", [_SwiGLU, _Packed])
@pytest.mark.parametrize("autocast", [False, True])
def test_swiglu_patterns_match_eager(cls, autocast):
    import autokernel
    torch.manual_seed(0)
    ref = nn.Sequential(cls()).to(DEV)
    opt = autokernel.optimize(copy.deepcopy(ref), training=True)
    assert len(autokernel.report(opt)["patterns"]) == 1
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
