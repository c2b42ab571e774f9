"""Cross-entropy CUDA kernels (rows + chunked linear) vs the oracle and golden fixtures."""
import pytest
import torch

from conftest import assert_fp32_close, assert_lowp_close, golden
from oracle import hot_path_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [("plain", {}), ("softcap", dict(softcap=5.0)), ("ls", dict(label_smoothing=0.1)),
         ("zloss", dict(z_loss_weight=1e-2)), ("all", dict(softcap=7.0, label_smoothing=0.05, z_loss_weight=1e-3))]


@pytest.mark.parametrize("mode", ["fused", "tiny"])
@pytest.mark.parametrize("case,kw", CASES)
def test_ce_full_golden_cuda(case, kw, mode):
    from kernels import ce_fused
    g = golden("ce")
    x = torch.from_numpy(g["logits"]).to(DEV).requires_grad_(True)
    t = torch.from_numpy(g["targets"]).to(DEV)
    loss = ce_fused.ce_full(x, t, mode=mode, **kw)
    ref = float(g[f"{case}_loss"])
    assert abs(loss.item() - ref) <= 1e-5 * max(1.0, abs(ref))
    loss.backward()
    assert_fp32_close(x.grad, g[f"{case}_grad"], what="grad")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,V", [(64, 32768), (7, 50257), (3, 1000), (5, 7)])
def test_ce_rows_kernel(dtype, B, V):
    from kernels import ce_fused
    g = torch.Generator().manual_seed(B + V)
    x = (torch.randn(B, V, generator=g) * 2).to(dtype)
    t = torch.randint(0, V, (B,), generator=g)
    t[0] = -100
    mod = ce_fused._get_fwd_module()
    losses, lse, rmax, rsum, grad = mod.cross_entropy_fwd_hip(x.to(DEV), t.to(DEV), 0.0, -100, 0.0, 1, 1, 0.5)
    rl, rlse, rg = O.ce_rows(x, t, scale=0.5)
    assert_fp32_close(losses, rl, rtol=1e-5 if dtype == torch.float32 else 1e-3, what="losses")
    assert_fp32_close(lse, rlse, rtol=1e-5 if dtype == torch.float32 else 1e-3, what="lse")
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(grad, rg, what="grad")
    g2 = ce_fused._get_bwd_module().cross_entropy_bwd_tiny_hip(x.to(DEV), t.to(DEV), rmax, rsum, 0.0, -100, 0.0, 0.5)
    (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(g2, rg, what="tiny grad")


def test_kernel_fn_and_facade():
    import kernel
    x = torch.randn(32, 4096, device=DEV, dtype=torch.bfloat16)
    t = torch.randint(0, 4096, (32,), device=DEV)
    ref = torch.nn.functional.cross_entropy(x.double().cpu(), t.cpu())
    assert abs(kernel.kernel_fn(x, t).item() - ref.item()) < 1e-3


def test_ce_all_ignored_gives_zero():
    from kernels import ce_fused
    x = torch.randn(4, 100, device=DEV, requires_grad=True)
    t = torch.full((4,), -100, device=DEV)
    loss = ce_fused.ce_full(x, t)
    loss.backward()
    assert loss.item() == 0.0 and torch.all(x.grad == 0)


def test_chunked_linear_ce_golden_cuda():
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    g = golden("linear_ce")
    H = torch.from_numpy(g["H"]).to(DEV).requires_grad_(True)
    W = torch.from_numpy(g["W"]).to(DEV).requires_grad_(True)
    lab = torch.from_numpy(g["labels"]).to(DEV)
    loss = ChunkedLinearCrossEntropyLoss(chunk_size=40)(H, W, lab)
    assert abs(loss.item() - float(g["loss"])) < 1e-4
    loss.backward()
    assert_fp32_close(H.grad, g["dH"], rtol=1e-4, what="dH")
    assert_fp32_close(W.grad, g["dW"], rtol=1e-4, what="dW")


@pytest.mark.parametrize("N,D,V", [(1024, 256, 32768), (300, 64, 1000)])
def test_chunked_linear_ce_bf16(N, D, V):
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    g = torch.Generator().manual_seed(N)
    H = torch.randn(N, D, generator=g).to(torch.bfloat16)
    W = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16)
    lab = torch.randint(0, V, (N,), generator=g)
    lab[::20] = -100
    Hc, Wc = H.to(DEV).requires_grad_(True), W.to(DEV).requires_grad_(True)
    loss = ChunkedLinearCrossEntropyLoss(chunk_size=256)(Hc, Wc, lab.to(DEV))
    rl, rdh, rdw = O.linear_ce(H, W, lab)
    assert abs(loss.item() - rl.item()) < 2e-2
    loss.backward()
    assert_lowp_close(Hc.grad, rdh, what="dH")
    assert_lowp_close(Wc.grad, rdw, what="dW")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N,D,V", [(1024, 256, 32768), (200, 72, 1000), (384, 768, 50304), (8, 64, 8)])
def test_fused_tcgen05_linear_ce(dtype, N, D, V):
    from kernels import _ak
    g = torch.Generator().manual_seed(N + D + V)
    H = torch.randn(N, D, generator=g).to(dtype)
    W = (torch.randn(V, D, generator=g) * 0.05).to(dtype)
    lab = torch.randint(0, V, (N,), generator=g)
    lab[::7] = -100
    loss, lse, dH, dW = _ak.linear_ce_fwdbwd(H.to(DEV), W.to(DEV), lab.to(DEV), -100)
    rl, rdh, rdw = O.linear_ce(H, W, lab)
    logits = H.double() @ W.double().t()
    assert_fp32_close(lse, torch.logsumexp(logits, -1), rtol=2e-4, what="lse")
    assert abs(loss.item() - rl.item()) <= 2e-3 * max(1.0, abs(rl.item()))
    assert_lowp_close(dH, rdh, what="dH")
    assert_lowp_close(dW, rdw, what="dW")


def test_fused_linear_ce_module_autograd():
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    g = torch.Generator().manual_seed(0)
    H = torch.randn(512, 128, generator=g).to(torch.bfloat16)
    W = (torch.randn(4096, 128, generator=g) * 0.05).to(torch.bfloat16)
    lab = torch.randint(0, 4096, (512,), generator=g)
    Hc, Wc = H.to(DEV).requires_grad_(True), W.to(DEV).requires_grad_(True)
    loss = ChunkedLinearCrossEntropyLoss()(Hc, Wc, lab.to(DEV))
    (2.0 * loss).backward()
    rl, rdh, rdw = O.linear_ce(H, W, lab)
    assert abs(loss.item() - rl.item()) < 2e-3 * abs(rl.item())
    assert_lowp_close(Hc.grad, 2 * rdh, what="dH")
    assert_lowp_close(Wc.grad, 2 * rdw, what="dW")


@pytest.mark.parametrize("N,D,V", [(1024, 256, 32768), (200, 72, 1000), (8, 64, 8)])
def test_linear_ce_logits_grad(N, D, V):
    from kernels import _ak
    g = torch.Generator().manual_seed(N + V)
    H = torch.randn(N, D, generator=g).to(torch.bfloat16)
    W = (torch.randn(V, D, generator=g) * 0.05).to(torch.bfloat16)
    lab = torch.randint(0, V, (N,), generator=g)
    lab[::5] = -100
    loss, lse, G = _ak.linear_ce_logits_grad(H.to(DEV), W.to(DEV), lab.to(DEV), -100)
    x = H.double() @ W.double().t()
    n = (lab != -100).sum().item()
    _, rlse, rg = O.ce_rows(x, lab, scale=1.0 / n)
    assert_fp32_close(lse, rlse, rtol=2e-3, what="lse")
    assert_lowp_close(G.float() * n, rg * n, what="G")
    rl, _, _ = O.linear_ce(H, W, lab)
    assert abs(loss.item() - rl.item()) <= 3e-3 * max(1.0, abs(rl.item()))


@pytest.mark.parametrize("use_fused", [True, False])
def test_linear_ce_upstream_grad_scaling_on_device(use_fused):
    """The precomputed dH / dW are scaled by the upstream gradient on the device (no
    grad_output.item()): exactly the unit-gradient result times the scale, unchanged for a unit
    gradient, and a second backward through the same graph is refused."""
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    g = torch.Generator().manual_seed(5)
    H = torch.randn(300, 64, generator=g).to(torch.bfloat16).to(DEV)
    W = (0.02 * torch.randn(1000, 64, generator=g)).to(torch.bfloat16).to(DEV)
    lab = torch.randint(0, 1000, (300,), generator=g).to(DEV)
    mod = ChunkedLinearCrossEntropyLoss(chunk_size=128)
    mod.use_fused = use_fused
    grads = []
    for scale in (1.0, 2.5):
        h, w = H.clone().requires_grad_(True), W.clone().requires_grad_(True)
        loss = mod(h, w, lab)
        loss.backward(torch.tensor(scale, device=DEV))
        grads.append((h.grad.float(), w.grad.float()))
    assert torch.equal(grads[1][0], (grads[0][0].to(torch.bfloat16) * 2.5).float()) or \
        torch.allclose(grads[1][0], grads[0][0] * 2.5, rtol=1e-2, atol=1e-6)
    torch.testing.assert_close(grads[1][1], grads[0][1] * 2.5, rtol=1e-2, atol=1e-6)
    h, w = H.clone().requires_grad_(True), W.clone().requires_grad_(True)
    loss = mod(h, w, lab)
    loss.backward(retain_graph=True)
    with pytest.raises(RuntimeError, match="twice"):
        loss.backward()


def _fp32_linear_ce(H, W, lab, ignore_index=-100):
    """loss, lse, dH, dW of mean CE(H W^T) in fp32 on the GPU (the float64 oracle's formulas)."""
    Hf = H.float().requires_grad_(True)
    Wf = W.float().requires_grad_(True)
    lg = Hf @ Wf.t()
    loss = torch.nn.functional.cross_entropy(lg, lab, ignore_index=ignore_index)
    loss.backward()
    return loss.detach(), torch.logsumexp(lg.detach(), -1), Hf.grad, Wf.grad


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_ce_several_chunks_ragged(dtype):
    """N above one 16384-row chunk with a ragged last chunk (dW accumulated in fp32 across chunks,
    the last chunk adds and rounds), V not a multiple of the 64-deep K block nor of the 256-wide tile."""
    from kernels import _ak
    g = torch.Generator().manual_seed(11)
    N, D, V = 16384 + 520, 128, 4000
    H = torch.randn(N, D, generator=g).to(dtype).to(DEV)
    W = (torch.randn(V, D, generator=g) * 0.05).to(dtype).to(DEV)
    lab = torch.randint(0, V, (N,), generator=g)
    lab[::9] = -100
    lab = lab.to(DEV)
    loss, lse, dH, dW = _ak.linear_ce_fwdbwd(H, W, lab, -100)
    _ak.check_status()
    rl, rlse, rdh, rdw = _fp32_linear_ce(H, W, lab)
    n = (lab != -100).sum().item()
    assert abs(loss.item() - rl.item()) <= 2e-3 * max(1.0, abs(rl.item()))
    torch.testing.assert_close(lse, rlse, rtol=0, atol=3e-2)
    assert_lowp_close(dH.float() * n, rdh * n, what="dH*n")
    assert_lowp_close(dW.float() * n, rdw * n, what="dW*n")


def test_linear_ce_row_shards_with_global_valid_count():
    """Rows split over two shards, each call given 1 / (valid rows of both): the loss and dW of
    the shards sum to the unsharded ones and dH concatenates (what the multi-GPU path all-reduces)."""
    from kernels import _ak
    g = torch.Generator().manual_seed(12)
    N, D, V = 2048, 256, 8192
    H = torch.randn(N, D, generator=g).to(torch.bfloat16).to(DEV)
    W = (torch.randn(V, D, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    lab = torch.randint(0, V, (N,), generator=g)
    lab[::13] = -100
    lab = lab.to(DEV)
    loss, _, dH, dW = _ak.linear_ce_fwdbwd(H, W, lab)
    inv = (1.0 / (lab != -100).sum().float()).reshape(1)
    parts = [_ak.linear_ce_fwdbwd(H[s], W, lab[s], inv_valid=inv) for s in (slice(0, 1000), slice(1000, N))]
    _ak.check_status()
    torch.testing.assert_close(parts[0][0] + parts[1][0], loss, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(torch.cat([parts[0][2], parts[1][2]]).float(), dH.float(), rtol=0, atol=1e-6)
    torch.testing.assert_close(parts[0][3].float() + parts[1][3].float(), dW.float(), rtol=2e-2, atol=1e-5)


@pytest.mark.parametrize("a_t,b_t", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (296, 136, 200), (1000, 520, 1032), (8, 8, 8)])
def test_tc_gemm_layouts(a_t, b_t, M, N, K):
    """The tcgen05 GEMM for all four operand layouts (K-contiguous or M / N-contiguous), ragged
    M, N and K, against an fp32 GEMM of the same bf16 inputs."""
    from kernels import _ak
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    b = torch.randn(K, N, generator=g).to(torch.bfloat16).to(DEV)
    aa = a.t().contiguous().t() if a_t else a   # same values, M-contiguous storage
    bb = b.t().contiguous().t() if not b_t else b  # b_t: N-contiguous [K][N]; else K-contiguous
    c = _ak.tc_gemm(aa, bb, out_dtype=torch.float32)
    _ak.check_status()
    ref = a.float() @ b.float()
    torch.testing.assert_close(c, ref, rtol=1e-4, atol=1e-3)
