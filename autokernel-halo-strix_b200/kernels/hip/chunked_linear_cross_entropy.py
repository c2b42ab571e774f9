"""Chunked linear + cross-entropy on B200 (logits never materialised in full).

Drop-in for kernels/hip/chunked_linear_cross_entropy.py of the reference
(`ChunkedLinearCrossEntropyLoss`, :178-229; `_ChunkedLinearCrossEntropy`,
:50-175): for each row chunk, logits = h W^T, the fused CE row kernel writes
loss, lse and the pre-scaled gradient G, then dH = G W and dW += G^T h (fp32
accumulation).  All gradients are produced in the forward; the backward
returns them scaled by grad_output.

For bf16/fp16 inputs without softcap, label smoothing or z-loss the whole
computation is one call into the library (`ak_linear_ce_fwdbwd`), and all three
contractions run on its tcgen05 GEMM: per chunk of at most 16384 rows the logits
GEMM reduces its tiles to softmax statistics and keeps that chunk's 16-bit
logits, which become G = softmax - onehot in place and feed dW += G^T h and
dH = G W in one grouped GEMM launch (1 / n_valid is applied to the fp32
accumulators in the GEMM epilogue).  Full [N, V] logits are
never stored and no cuBLAS GEMM runs.  Other feature combinations use the
row-chunked path below (cuBLAS GEMMs around the fused CE row kernel).

Differences, all deliberate: inputs keep their dtype (the reference coerces to
fp16, :219-223); the valid-row count and 1/n_valid stay on the device (the
reference syncs with `.item()`, :73).
"""
import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.amp import custom_bwd, custom_fwd

from kernels import _ak


class _ChunkedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, hidden, weight, targets, chunk_size, softcap, ignore_index, label_smoothing, z_loss_weight):
        N, D = hidden.shape
        V = weight.shape[0]
        dev = hidden.device
        h = hidden.contiguous()
        w = weight.to(h.dtype).contiguous()
        t = targets.contiguous()
        inv_valid = _ak.ce_inv_valid(t, ignore_index)
        losses = torch.empty(N, dtype=torch.float32, device=dev)
        lse = torch.empty(N, dtype=torch.float32, device=dev)
        grad_h = torch.empty_like(h) if hidden.requires_grad else None
        grad_w = torch.zeros(V, D, dtype=torch.float32, device=dev) if weight.requires_grad else None
        for s in range(0, N, chunk_size):
            e = min(s + chunk_size, N)
            logits = F.linear(h[s:e], w)
            if z_loss_weight > 0:
                # z-loss gradient 2 w lse softmax / n_valid needs the final lse: two passes.
                lc, zc, rm, rs, _ = _ak.ce_rows_fwd(logits, t[s:e], softcap, ignore_index, label_smoothing,
                                                    save_max_sum=True)
                g = _ak.ce_rows_bwd(logits, t[s:e], rm, rs, softcap, ignore_index, label_smoothing, scale=1.0,
                                    scale_dev=inv_valid, z_coef=2.0 * z_loss_weight, out=logits)
            else:
                lc, zc, _, _, g = _ak.ce_rows_fwd(logits, t[s:e], softcap, ignore_index, label_smoothing,
                                                  write_grad=True, scale_grad=1.0, scale_dev=inv_valid)
            losses[s:e] = lc
            lse[s:e] = zc
            if grad_h is not None:
                torch.mm(g, w, out=grad_h[s:e])
            if grad_w is not None:
                grad_w += torch.mm(g.t(), h[s:e], out_dtype=torch.float32)
        loss, _ = _ak.ce_rows_reduce(losses, lse, t, ignore_index, z_loss_weight)
        ctx.save_for_backward(grad_h, grad_w.to(weight.dtype) if grad_w is not None else None)
        ctx.req = (hidden.requires_grad, weight.requires_grad)
        return loss

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        gh, gw = _take_saved(ctx)
        return (_scaled(gh, grad_output) if ctx.req[0] else None), (_scaled(gw, grad_output) if ctx.req[1] else None), \
            None, None, None, None, None, None


def _take_saved(ctx):
    """The gradients precomputed in the forward.  They are scaled in place, so a second
    backward through the same graph (retain_graph=True) is refused instead of returning
    twice-scaled values."""
    if getattr(ctx, "consumed", False):
        raise RuntimeError("fused linear + cross-entropy: backward through the same graph twice is not supported "
                           "(the gradients are computed in the forward and consumed by the first backward)")
    ctx.consumed = True
    return ctx.saved_tensors


def _scaled(g, grad_output):
    """The saved gradient times the scalar upstream gradient.  The reference checks
    `grad_output.item() == 1.0` on the host to skip the multiply
    (chunked_linear_cross_entropy.py:159-169); here the scalar is read on the device by the
    scaling kernel itself (nothing written when it is 1), so there is no host sync and the
    backward can be captured in a CUDA graph.  The saved tensor is owned by this call (made in
    the forward, used once), so it is scaled in place."""
    if g is None:
        return None
    if grad_output.numel() != 1:
        return g * grad_output.to(g.dtype)
    return _ak.scale_by_device_scalar_(g, grad_output)


class _FusedLinearCrossEntropy(torch.autograd.Function):
    """tcgen05 path: loss, dH and dW come out of one C-ABI call (all GEMMs on our kernel)."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, hidden, weight, targets, ignore_index):
        w = weight.to(hidden.dtype).contiguous()
        h = hidden.contiguous()
        loss, _lse, dh, dw = _ak.linear_ce_fwdbwd(h, w, targets, ignore_index, need_dh=hidden.requires_grad,
                                                  need_dw=weight.requires_grad)
        ctx.save_for_backward(dh, dw.to(weight.dtype) if dw is not None else None)
        ctx.req = (hidden.requires_grad, weight.requires_grad)
        return loss

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        gh, gw = _take_saved(ctx)
        return (_scaled(gh, grad_output) if ctx.req[0] else None), \
            (_scaled(gw, grad_output) if ctx.req[1] else None), None, None


class ChunkedLinearCrossEntropyLoss(nn.Module):
    """`nn.Linear + nn.CrossEntropyLoss` without materialising all logits.

    Args mirror the reference: chunk_size, softcap, ignore_index, label_smoothing, z_loss_weight.
    forward(hidden (N, D) or (B, T, D), weight (V, D), targets (N,) or (B, T)) -> scalar mean loss.
    """

    def __init__(self, chunk_size: int = 512, softcap: float = 0.0, ignore_index: int = -100,
                 label_smoothing: float = 0.0, z_loss_weight: float = 0.0):
        super().__init__()
        self.chunk_size = int(chunk_size)
        self.softcap = float(softcap)
        self.ignore_index = int(ignore_index)
        self.label_smoothing = float(label_smoothing)
        self.z_loss_weight = float(z_loss_weight)
        # tcgen05 fused kernel for bf16/fp16 without softcap / smoothing / z-loss
        self.use_fused = True

    def forward(self, hidden, weight, targets):
        if hidden.dim() == 3:
            hidden = hidden.reshape(-1, hidden.shape[-1])
        if targets.dim() == 2:
            targets = targets.reshape(-1)
        if (self.use_fused and self.softcap == 0.0 and self.label_smoothing == 0.0 and self.z_loss_weight == 0.0
                and hidden.is_cuda and _ak.linear_ce_supported(hidden, weight.to(hidden.dtype))):
            return _FusedLinearCrossEntropy.apply(hidden, weight, targets, self.ignore_index)
        return _ChunkedLinearCrossEntropy.apply(hidden, weight, targets, self.chunk_size, self.softcap,
                                                self.ignore_index, self.label_smoothing, self.z_loss_weight)
