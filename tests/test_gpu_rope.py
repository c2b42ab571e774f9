"""Rotary embedding CUDA kernels vs the CPU oracle and the golden fixtures
(reference: kernels/hip/rotary_embedding.py, autokernel::rotary_emb_fp32 in
kernels/hip/_torch_ops.py:112-169, FusedQKVPattern _patterns.py:216-361,488-505)."""
import copy

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


def tables(N, D, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    ang = torch.outer(torch.arange(N, dtype=torch.float32), inv)
    return ang.cos(), ang.sin()


def test_rope_golden_cuda():
    from kernels.hip import rotary_embedding, rotary_embedding_backward
    g = golden("rope")
    x, c, s, dy = (torch.from_numpy(g[k]).to(DEV) for k in ("x", "cos", "sin", "dy"))
    assert_fp32_close(rotary_embedding.kernel_fn_fp32(x, c, s), g["y"], what="y")
    assert_fp32_close(rotary_embedding.kernel_fn(x, c, s), g["y_ref"], what="y")
    assert_fp32_close(rotary_embedding_backward.kernel_fn(dy, c, s), g["dx_autograd"], what="dx")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,N,D", [(2, 12, 1024, 64), (1, 3, 17, 128), (2, 2, 5, 6), (1, 1, 1, 2), (3, 4, 33, 40)])
def test_rope_fwd_bwd(dtype, B, H, N, D):
    from kernels import _ak
    g = torch.Generator().manual_seed(B + H + N + D)
    x = torch.randn(B, H, N, D, generator=g).to(dtype)
    dy = torch.randn(B, H, N, D, generator=g).to(dtype)
    c, s = tables(N, D)
    close(dtype, _ak.rope_fwd(x.to(DEV), c.to(DEV), s.to(DEV)), O.rope(x, c, s), "y")
    close(dtype, _ak.rope_bwd(dy.to(DEV), c.to(DEV), s.to(DEV)), O.rope_bwd(dy, c, s), "dx")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_strided_views_of_packed_qkv(dtype):
    """q and k read straight from a (B, T, W) fused projection, written head-major."""
    from kernels import _ak
    B, T, H, KH, hd = 2, 77, 12, 4, 64
    qkv = torch.randn(B, T, (H + 2 * KH) * hd, device=DEV).to(dtype)
    q = qkv[..., :H * hd].view(B, T, H, hd).transpose(1, 2)
    k = qkv[..., H * hd:(H + KH) * hd].view(B, T, KH, hd).transpose(1, 2)
    c, s = tables(T, hd)
    for t in (q, k):
        y = _ak.rope_fwd(t, c.to(DEV), s.to(DEV))
        assert y.is_contiguous() and y.shape == t.shape
        close(dtype, y, O.rope(t.cpu(), c, s), "y")


def test_rope_roundtrip_and_table_checks():
    from kernels import _ak
    x = torch.randn(2, 4, 300, 64, device=DEV)
    c, s = tables(300, 64)
    c, s = c.to(DEV), s.to(DEV)
    assert_fp32_close(_ak.rope_bwd(_ak.rope_fwd(x, c, s), c, s), x, rtol=1e-5, what="inverse rotation")
    with pytest.raises(ValueError):
        _ak.rope_fwd(x, torch.ones(300, 64, device=DEV), torch.ones(300, 64, device=DEV))  # full-width tables
    with pytest.raises(ValueError):
        _ak.rope_fwd(x, c[:10], s[:10])  # too few positions


@pytest.mark.parametrize("under_autocast", [False, True])
def test_rotary_custom_op_autograd(under_autocast):
    import kernels.hip._torch_ops  # noqa: F401
    x = torch.randn(2, 8, 128, 64, device=DEV, dtype=torch.float16, requires_grad=True)
    c, s = tables(128, 64)
    with torch.amp.autocast(device_type="cuda", dtype=torch.float16, enabled=under_autocast):
        y = torch.ops.autokernel.rotary_emb_fp32(x, c.to(DEV), s.to(DEV))
    assert y.dtype == (torch.float32 if under_autocast else torch.float16)  # autocast rule: fp32
    dy = torch.randn(y.shape, device=DEV, dtype=y.dtype)
    y.backward(dy)
    close(y.dtype, y, O.rope(x.detach().cpu(), c, s), "y")
    assert_lowp_close(x.grad, O.rope_bwd(dy.cpu(), c, s), what="dx")


@pytest.mark.parametrize("autocast", [False, True])
def test_fused_qkv_pattern_matches_eager(autocast):
    import autokernel
    from halo_training.hybrid_lm import GQAAttention, HybridConfig
    torch.manual_seed(0)
    ref = nn.Sequential(GQAAttention(HybridConfig())).to(DEV)
    opt = autokernel.optimize(copy.deepcopy(ref), training=True)
    assert autokernel.report(opt)["patterns"]["fused_qkv"]["modules_replaced"] == 1
    x = torch.randn(2, 256, 768, device=DEV)
    outs = []
    for m in (ref, opt):
        xi = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            y = m(xi)
        y.float().square().mean().backward()
        outs.append((y.float(), xi.grad, {n: p.grad for n, p in m.named_parameters()}))
    tol = dict(atol=3e-2, rtol=3e-2) if autocast else dict(atol=2e-4, rtol=2e-4)
    torch.testing.assert_close(outs[1][0], outs[0][0], **tol)
    torch.testing.assert_close(outs[1][1], outs[0][1], **tol)
    assert set(outs[1][2]) == set(outs[0][2])
    for n, g in outs[0][2].items():
        torch.testing.assert_close(outs[1][2][n].float(), g.float(), **tol, msg=n)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 6])  # vector path and the pair path
def test_rope_strided_modes(dtype, D):
    """ak_rope_strided: strided input and output, rotate / inverse / copy, bit-exact against
    the dense kernels (same fp32 arithmetic) and untouched bytes outside the written slice."""
    from kernels import _ak
    B, H, N = 2, 3, 40
    c, s = (t.to(DEV) for t in tables(N, D))
    src = torch.randn(B, N, 5 * H * D, device=DEV).to(dtype)
    x = src[..., H * D:2 * H * D].view(B, N, H, D).transpose(1, 2)
    for mode, ref in ((1, _ak.rope_fwd(x, c, s)), (-1, _ak.rope_bwd(x, c, s)), (0, x.contiguous())):
        dst = torch.full((B, N, 3 * H * D), 7.0, device=DEV).to(dtype)
        y = dst[..., H * D:2 * H * D].view(B, N, H, D).transpose(1, 2)
        _ak.rope_into(y, x, c, s, mode)
        assert torch.equal(y, ref), mode
        assert torch.all(dst[..., :H * D] == 7) and torch.all(dst[..., 2 * H * D:] == 7)
    with pytest.raises(ValueError):
        _ak.rope_into(y, x, c, s, 2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_qkv_rope_split_matches_separate_ops(dtype):
    """qkv_rope_split: forward equals rope of the q / k slices and the v slice; backward
    equals the gradient of that composition (bit-exact: the same kernels and arithmetic), in one
    packed d(qkv)."""
    from kernels import _ak
    from kernels.hip._torch_ops import qkv_rope_split
    B, T, H, KH, hd = 2, 96, 12, 4, 64
    c, s = (t.to(DEV) for t in tables(T, hd))
    qkv = torch.randn(B, T, (H + 2 * KH) * hd, device=DEV).to(dtype).requires_grad_(True)
    q, k, v = qkv_rope_split(qkv, c, s, H, KH)
    assert q.shape == (B, H, T, hd) and k.shape == (B, KH, T, hd) and v.shape == (B, KH, T, hd)
    qs, ks = H * hd, KH * hd
    raw = qkv.detach()
    assert torch.equal(q, _ak.rope_fwd(raw[..., :qs].view(B, T, H, hd).transpose(1, 2), c, s))
    assert torch.equal(k, _ak.rope_fwd(raw[..., qs:qs + ks].view(B, T, KH, hd).transpose(1, 2), c, s))
    assert torch.equal(v, raw[..., qs + ks:].view(B, T, KH, hd).transpose(1, 2))
    gq, gk, gv = (torch.randn_like(t) for t in (q, k, v))
    torch.autograd.backward((q, k, v), (gq, gk, gv))
    want = torch.cat([_ak.rope_bwd(gq, c, s).transpose(1, 2).reshape(B, T, qs),
                      _ak.rope_bwd(gk, c, s).transpose(1, 2).reshape(B, T, ks),
                      gv.transpose(1, 2).reshape(B, T, ks)], dim=-1)
    assert torch.equal(qkv.grad, want)
    # only q used: the k and v columns of the gradient are zero
    qkv.grad = None
    q, k, v = qkv_rope_split(qkv, c, s, H, KH)
    q.backward(gq)
    assert torch.equal(qkv.grad[..., :qs], want[..., :qs]) and torch.all(qkv.grad[..., qs:] == 0)
