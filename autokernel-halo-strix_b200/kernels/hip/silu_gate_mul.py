"""SiLU gate multiply (SwiGLU body) forward on B200: y = silu(gate) * up.

Drop-in for kernels/hip/silu_gate_mul.py of the reference (`kernel_fn(gate,
up)`, :102-118).  The reference runs its kernel for fp16 only and uses
`F.silu(gate) * up` otherwise; here fp32, bf16 and fp16 all run the CUDA kernel
(fp32 arithmetic, one rounding).  gate and up may be strided row views, e.g. the
two halves of one packed `w_gate_up` projection, without a copy.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "silu_gate_mul"
BACKEND = "cuda_sm100a"


def kernel_fn(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    assert gate.is_cuda and up.is_cuda
    return _ak.silu_gate_mul_fwd(gate, up)
