"""Collapsed (single-state) selective scan forward on B200, fp32.

Drop-in for kernels/hip/selective_scan.py (`kernel_fn`, selective_scan.py:214-241):
    state[t] = dA[t] * state[t-1] + dBx[t]
    y[t]     = C[t] * state[t] + D * x[t]
dA, dBx, C, x: (batch, seq, d_inner) fp32; D: (d_inner,) fp32.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "selective_scan"
BACKEND = "cuda_sm100a"


def kernel_fn(dA: torch.Tensor, dBx: torch.Tensor, C: torch.Tensor, D: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    assert dA.is_cuda and dA.dtype == torch.float32
    return _ak.scan1_fwd(dA, dBx, C, D, x)
