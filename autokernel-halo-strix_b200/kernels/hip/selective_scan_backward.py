"""Collapsed selective scan backward on B200, fp32.

Drop-in for kernels/hip/selective_scan_backward.py (`kernel_fn`,
selective_scan_backward.py:393-421); gradients as in the sequential autograd
fallback kernels/hip/_torch_ops.py:353-389.  Returns
(grad_dA, grad_dBx, grad_C, grad_D, grad_x), all fp32; grad_D is reduced
deterministically (no atomics).
"""
import torch

from kernels import _ak

KERNEL_TYPE = "selective_scan_backward"
BACKEND = "cuda_sm100a"


def kernel_fn(dA, dBx, C, D, x, grad_y) -> tuple:
    assert dA.is_cuda and dA.dtype == torch.float32
    return _ak.scan1_bwd(dA, dBx, C, D, x, grad_y.float())
