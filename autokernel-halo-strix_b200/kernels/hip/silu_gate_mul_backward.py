"""SiLU gate multiply backward on B200.

Drop-in for kernels/hip/silu_gate_mul_backward.py of the reference
(`kernel_fn(gate, up, grad_output) -> (grad_gate, grad_up)`, :145-180):
grad_gate = dy * up * sigmoid(g) * (1 + g * (1 - sigmoid(g))),
grad_up = dy * silu(g), in one pass for every dtype.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "silu_gate_mul_backward"
BACKEND = "cuda_sm100a"


def kernel_fn(gate: torch.Tensor, up: torch.Tensor, grad_output: torch.Tensor):
    assert gate.is_cuda and up.is_cuda and grad_output.is_cuda
    return _ak.silu_gate_mul_bwd(gate, up, grad_output)
