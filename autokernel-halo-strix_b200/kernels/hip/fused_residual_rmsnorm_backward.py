"""Fused residual + RMSNorm backward on B200.

Drop-in for kernels/hip/fused_residual_rmsnorm_backward.py of the reference
(`kernel_fn(hidden, weight, grad_hidden, grad_normed)` -> (grad_x,
grad_residual, grad_weight), :248-300): grad_x = grad_residual = grad_hidden +
the RMSNorm backward of grad_normed, grad_weight = sum over rows of
grad_normed * hidden * rstd (fp32 accumulation, returned in weight's dtype as
the reference does).  One kernel pass over hidden, grad_hidden and grad_normed;
grad_weight is reduced deterministically (no atomics).
"""
import torch

from kernels import _ak

KERNEL_TYPE = "fused_residual_rmsnorm_backward"
BACKEND = "cuda_sm100a"

EPS = 1e-6


def kernel_fn(hidden: torch.Tensor, weight: torch.Tensor, grad_hidden: torch.Tensor, grad_normed: torch.Tensor,
              eps: float = EPS):
    assert hidden.is_cuda
    dx, dw = _ak.fused_res_rmsnorm_bwd(hidden, weight, grad_hidden, grad_normed, eps)
    return dx, dx, dw.to(weight.dtype)
