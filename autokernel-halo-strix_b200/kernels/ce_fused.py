"""Fused cross-entropy over logit rows on B200 (online softmax, one pass).

Drop-in for the reference's kernels/ce_fused.py: same module constants
(KERNEL_TYPE, MODEL_SHAPES, TEST_SIZES, TOLERANCES, FLOPS_FN, BYTES_FN), same
`kernel_fn(logits, targets)`, `ce_full(...)`, `_CrossEntropyHIP` autograd
Function and the `_get_fwd_module().cross_entropy_fwd_hip(...)` /
`_get_bwd_module().cross_entropy_bwd_tiny_hip(...)` call contracts
(ce_fused.py:333-382, 490-522, 529-554, 557-785).

Differences, all deliberate:
  * the kernel runs natively for fp32, bf16 and fp16 (the reference casts to
    fp16, ce_fused.py:705-709, or falls back to PyTorch for fp32);
  * the valid-row count and the loss mean are reduced on the device; the
    gradient scale 1/n_valid is read by the kernel from device memory, so the
    forward has no host sync (the reference calls `.item()`, ce_fused.py:604).
"""
import torch

from kernels import _ak

KERNEL_TYPE = "cross_entropy"
BACKEND = "cuda_sm100a"

MODEL_SHAPES = {'batch': 4096, 'vocab': 32768}

TEST_SIZES = [
    ("model_primary", {'batch': 4096, 'vocab': 32768}),
    ("model_half", {'batch': 2048, 'vocab': 16384}),
    ("model_double", {'batch': 8192, 'vocab': 65536}),
]

TOLERANCES = {'float16': {'atol': 0.01, 'rtol': 0.01}, 'bfloat16': {'atol': 0.02, 'rtol': 0.02},
              'float32': {'atol': 1e-05, 'rtol': 1e-05}}


def FLOPS_FN(s):
    return 4 * s["batch"] * s["vocab"]


def BYTES_FN(s, dt_bytes):
    return (s["batch"] * s["vocab"] + s["batch"]) * dt_bytes


class _FwdModule:
    """Stand-in for the compiled forward extension of the reference."""

    @staticmethod
    def cross_entropy_fwd_hip(logits, targets, softcap, ignore_index, label_smoothing, write_grad, save_max_sum,
                              scale_grad):
        """Returns [losses, logsumexp, row_max, row_sum, grad_logits]; absent outputs are None."""
        if logits.dim() != 2:
            raise RuntimeError("logits must be [batch, vocab]")
        return _ak.ce_rows_fwd(logits, targets, float(softcap), int(ignore_index), float(label_smoothing),
                               write_grad=bool(write_grad), save_max_sum=bool(save_max_sum),
                               scale_grad=float(scale_grad))


class _BwdModule:
    """Stand-in for the compiled tiny-mode backward extension of the reference."""

    @staticmethod
    def cross_entropy_bwd_tiny_hip(logits, targets, row_maxes, row_sums, softcap, ignore_index, label_smoothing,
                                   scale_grad):
        return _ak.ce_rows_bwd(logits, targets, row_maxes, row_sums, float(softcap), int(ignore_index),
                               float(label_smoothing), float(scale_grad))


_fwd_module = _FwdModule()
_bwd_module = _BwdModule()


def _get_fwd_module():
    return _fwd_module


def _get_bwd_module():
    return _bwd_module


class _CrossEntropyHIP(torch.autograd.Function):
    """CE with online softmax; `mode="fused"` writes the gradient in the forward,
    `mode="tiny"` saves only (row_max, row_sum) and recomputes in the backward.
    `z_loss_weight > 0` adds w * mean(lse^2) over valid rows (forces tiny mode).
    Returns the mean loss over non-ignored rows, and per-row lse if return_z.
    """

    @staticmethod
    def forward(ctx, logits, targets, softcap, ignore_index, label_smoothing, mode, return_z, z_loss_weight=0.0):
        z_loss_weight = float(z_loss_weight)
        if z_loss_weight > 0.0 and mode != "tiny":
            mode = "tiny"
        fused = mode == "fused"
        ignore = -100 if ignore_index is None else int(ignore_index)
        inv_valid = _ak.ce_inv_valid(targets, ignore) if ignore_index is not None else torch.full(
            (), 1.0 / max(1, targets.numel()), dtype=torch.float32, device=logits.device)
        losses, lse, row_max, row_sum, grad = _ak.ce_rows_fwd(
            logits, targets, float(softcap), ignore, float(label_smoothing), write_grad=fused,
            save_max_sum=not fused, scale_grad=1.0, scale_dev=inv_valid if fused else None)
        loss, n_valid = _ak.ce_rows_reduce(losses, lse, targets, ignore, z_loss_weight)
        ctx.mode = mode
        ctx.softcap = float(softcap)
        ctx.ignore_index = ignore
        ctx.label_smoothing = float(label_smoothing)
        ctx.z_loss_weight = z_loss_weight
        if fused:
            ctx.save_for_backward(grad)
        else:
            ctx.save_for_backward(logits, targets, row_max, row_sum, inv_valid)
        if return_z:
            ctx.mark_non_differentiable(lse)
            return loss, lse
        return loss

    @staticmethod
    def backward(ctx, grad_loss, *rest):
        if ctx.mode == "fused":
            (saved_grad,) = ctx.saved_tensors
            if grad_loss.dim() == 0 and grad_loss.item() == 1.0:
                return saved_grad, None, None, None, None, None, None, None
            return saved_grad * grad_loss.to(saved_grad.dtype), None, None, None, None, None, None, None
        logits, targets, row_max, row_sum, inv_valid = ctx.saved_tensors
        scale_dev = (grad_loss.to(torch.float32) * inv_valid).reshape(())
        grad_logits = _ak.ce_rows_bwd(logits, targets, row_max, row_sum, ctx.softcap, ctx.ignore_index,
                                      ctx.label_smoothing, scale=1.0, scale_dev=scale_dev,
                                      z_coef=2.0 * ctx.z_loss_weight)
        return grad_logits, None, None, None, None, None, None, None


def kernel_fn(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean CE over rows with target != -100 (reference.cross_entropy_ref semantics)."""
    assert logits.is_cuda and targets.is_cuda
    if not (logits.requires_grad and torch.is_grad_enabled()):
        losses, lse, _, _, _ = _ak.ce_rows_fwd(logits, targets, 0.0, -100, 0.0)
        loss, _ = _ak.ce_rows_reduce(losses, lse, targets, -100, 0.0)
        return loss
    return _CrossEntropyHIP.apply(logits, targets, 0.0, -100, 0.0, "fused", False, 0.0)


def ce_full(logits: torch.Tensor, targets: torch.Tensor, *, softcap: float = 0.0, ignore_index: int = -100,
            label_smoothing: float = 0.0, mode: str = "fused", return_z: bool = False, z_loss_weight: float = 0.0):
    """Full-featured CE: softcap, ignore_index, label smoothing, fused/tiny modes, z-loss."""
    assert logits.is_cuda and targets.is_cuda
    return _CrossEntropyHIP.apply(logits, targets, softcap, ignore_index, label_smoothing, mode, return_z,
                                  float(z_loss_weight))
