"""Parity at the exact BASELINE configurations, with an fp32 PyTorch computation on the GPU as the
checker (the float64 CPU oracle would take minutes at these sizes; it pins the same formulas on
the small cases of test_gpu_ce.py / test_gpu_rmsnorm_softmax.py).

* causal row softmax, config 3: all 196,608 x 2048 bf16 rows, forward and backward;
* fused linear + cross-entropy, config 2: N = 32768, D = 768, V = 50304 bf16 with 5 % of the
  labels ignored: loss, lse, dH, dW through the product module (`ChunkedLinearCrossEntropyLoss`)
  and through the C entry `ak_linear_ce_fwdbwd`.

The full selective-scan configuration is checked against the reference's own CUDA kernel in
test_gpu_mamba_comparator.py.  Tolerances: the bf16 bound of conftest (|a-b| <= 0.02 + 0.02|b|)
on O(1) quantities; gradients of the mean loss are compared after multiplying by n_valid so the
bound applies to per-row quantities of order one.
"""
import pytest
import torch
import torch.nn.functional as F

from conftest import assert_lowp_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _causal_scores(rows, cols, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    s = (torch.randn(rows, cols, device=DEV, generator=g) / 8).to(torch.bfloat16)
    r = torch.arange(rows, device=DEV) % cols
    s.masked_fill_(torch.arange(cols, device=DEV)[None, :] > r[:, None], float("-inf"))
    dy = torch.randn(rows, cols, device=DEV, generator=g).to(torch.bfloat16)
    return s, dy


def test_softmax_causal_all_baseline_rows():
    from kernels import _ak
    from kernels.hip import softmax as sm
    rows, cols = 96 * 2048, 2048
    s, dy = _causal_scores(rows, cols, seed=3)
    y = sm.kernel_fn(s)
    dx = _ak.softmax_bwd(y, dy)
    masked = torch.arange(cols, device=DEV)[None, :] > (torch.arange(rows, device=DEV) % cols)[:, None]
    assert torch.all(y[masked] == 0) and torch.all(dx[masked] == 0)
    step = 8192
    for r0 in range(0, rows, step):
        yr = torch.softmax(s[r0:r0 + step].float(), dim=-1)
        dyr = dy[r0:r0 + step].float()
        dxr = yr * (dyr - (dyr * yr).sum(-1, keepdim=True))
        assert_lowp_close(y[r0:r0 + step].float(), yr, what=f"y rows {r0}+")
        assert_lowp_close(dx[r0:r0 + step].float(), dxr, what=f"dx rows {r0}+")
    # every row sums to one (the rows past 65,535 included)
    torch.testing.assert_close(y.float().sum(-1), torch.ones(rows, device=DEV), rtol=0, atol=2e-2)


def _linear_ce_inputs(N=32768, D=768, V=50304, seed=0):
    g = torch.Generator().manual_seed(seed)
    H = torch.randn(N, D, generator=g).to(torch.bfloat16)
    W = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16)
    lab = torch.randint(0, 50257, (N,), generator=g)
    lab[torch.randperm(N, generator=g)[: N // 20]] = -100
    return H.to(DEV), W.to(DEV), lab.to(DEV)


def _linear_ce_fp32_checker(H, W, lab, chunk=4096):
    """loss, lse, dH, dW of mean CE(H W^T) in fp32 on the GPU, row chunk by row chunk."""
    N = H.shape[0]
    Wf = W.float()
    valid = lab != -100
    n = valid.sum().item()
    lse = torch.empty(N, device=DEV)
    dH = torch.empty(N, W.shape[1], device=DEV)
    dW = torch.zeros_like(Wf)
    loss = 0.0
    for r0 in range(0, N, chunk):
        h = H[r0:r0 + chunk].float()
        lg = h @ Wf.t()
        l = torch.logsumexp(lg, -1)
        lse[r0:r0 + chunk] = l
        loss += F.cross_entropy(lg, lab[r0:r0 + chunk], ignore_index=-100, reduction="sum").item()
        G = torch.softmax(lg, -1)
        lr = lab[r0:r0 + chunk]
        vr = valid[r0:r0 + chunk]
        G[vr.nonzero().squeeze(1), lr[vr]] -= 1.0
        G[~vr] = 0.0
        dH[r0:r0 + chunk] = G @ Wf
        dW += G.t() @ h
        del lg, G
    return loss / n, lse, dH / n, dW / n, n


@pytest.fixture(scope="module")
def baseline_ce():
    H, W, lab = _linear_ce_inputs()
    ref = _linear_ce_fp32_checker(H, W, lab)
    return H, W, lab, ref


def _check_ce(loss, lse, dH, dW, ref, what):
    rloss, rlse, rdH, rdW, n = ref
    assert abs(float(loss) - rloss) <= 2e-3 * max(1.0, abs(rloss)), f"{what}: loss {float(loss)} vs {rloss}"
    if lse is not None:
        torch.testing.assert_close(lse.float(), rlse, rtol=0, atol=3e-2)
    assert_lowp_close(dH.float() * n, rdH * n, what=f"{what} dH*n_valid")
    assert_lowp_close(dW.float() * n, rdW * n, what=f"{what} dW*n_valid")


def test_linear_ce_baseline_shape_module(baseline_ce):
    from kernels import _ak
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    H, W, lab, ref = baseline_ce
    h, w = H.clone().requires_grad_(True), W.clone().requires_grad_(True)
    loss = ChunkedLinearCrossEntropyLoss()(h, w, lab)
    loss.backward()
    _ak.check_status()
    _check_ce(loss.item(), None, h.grad, w.grad, ref, "module")


def test_linear_ce_baseline_shape_c_entry(baseline_ce):
    from kernels import _ak
    H, W, lab, ref = baseline_ce
    loss, lse, dH, dW = _ak.linear_ce_fwdbwd(H, W, lab, -100)
    _ak.check_status()
    _check_ce(loss.item(), lse, dH, dW, ref, "ak_linear_ce_fwdbwd")
