"""Fused RMSNorm backward on B200.

Drop-in for kernels/hip/rmsnorm_backward.py (`kernel_fn`, rmsnorm_backward.py:239-281):
  grad_x      = rms_inv * (grad_out * w - normed * mean(grad_out * w * normed))
  grad_weight = sum over rows of grad_out * normed   (fp32)
The reference accumulates grad_weight with per-element global atomics
(rmsnorm_backward.py:176-177); here it is a deterministic two-stage column
reduction.  All of fp32 / bf16 / fp16 run on the GPU kernel.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "rmsnorm_backward"
BACKEND = "cuda_sm100a"

EPS = 1e-6


def kernel_fn(x: torch.Tensor, weight: torch.Tensor, grad_output: torch.Tensor, eps: float = EPS) -> tuple:
    """Returns (grad_x like x, grad_weight fp32 [N])."""
    assert x.is_cuda and weight.is_cuda and grad_output.is_cuda
    orig_shape = x.shape
    x2 = x.reshape(-1, x.shape[-1])
    g2 = grad_output.reshape(-1, grad_output.shape[-1])
    grad_x, grad_w = _ak.rmsnorm_bwd(x2, weight, g2, eps, dw_dtype=torch.float32)
    return grad_x.view(orig_shape), grad_w
