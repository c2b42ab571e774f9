"""RMSNorm forward on B200: y = x * rsqrt(mean(x^2) + eps) * weight.

Drop-in for kernels/hip/rmsnorm.py (reference `kernel_fn`, rmsnorm.py:156-177)
with the semantics of reference.rmsnorm_ref (reference.py:26-29).  Unlike the
reference, which runs its kernel only for fp16 and falls back to PyTorch for
fp32 (rmsnorm.py:160-163) or casts other dtypes to fp16 (:166-169), the CUDA
kernel here runs natively for fp32, bf16 and fp16 and returns x's dtype.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "rmsnorm"
BACKEND = "cuda_sm100a"

EPS = 1e-6


def kernel_fn(x: torch.Tensor, weight: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    """Entry point matching reference.rmsnorm_ref(x, weight); normalises the last dim."""
    assert x.is_cuda and weight.is_cuda
    return _ak.rmsnorm_fwd(x, weight, eps)
