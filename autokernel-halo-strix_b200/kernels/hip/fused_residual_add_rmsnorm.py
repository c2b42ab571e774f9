"""Fused residual add + RMSNorm forward on B200.

Drop-in for kernels/hip/fused_residual_add_rmsnorm.py of the reference:
  * `kernel_fn(x, residual, weight)` -> RMSNorm(x + residual) * weight
    (:340-374, semantics of reference.fused_residual_add_rmsnorm_ref,
    reference.py:72-78);
  * `kernel_fn_dual(x, residual, weight)` -> (hidden, normed) with
    hidden = x + residual (:377-418).
hidden is rounded to x's dtype before it is normalised, as the reference's
fp16 kernel does (`__hadd2`, then the fp32 norm of the rounded sum).  The
reference runs its kernel for fp16 only and casts or falls back to PyTorch
otherwise; here fp32, bf16 and fp16 all run the CUDA kernel and keep x's dtype.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "fused_residual_add_rmsnorm"
BACKEND = "cuda_sm100a"

EPS = 1e-6


def kernel_fn(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    assert x.is_cuda and residual.is_cuda and weight.is_cuda
    return _ak.fused_res_rmsnorm_fwd(x, residual, weight, eps, want_hidden=False)[1]


def kernel_fn_dual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = EPS):
    """Returns (hidden, normed)."""
    assert x.is_cuda and residual.is_cuda and weight.is_cuda
    return _ak.fused_res_rmsnorm_fwd(x, residual, weight, eps, want_hidden=True)
