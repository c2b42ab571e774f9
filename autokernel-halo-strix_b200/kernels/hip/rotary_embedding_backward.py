"""Rotary embedding backward on B200.

Drop-in for kernels/hip/rotary_embedding_backward.py of the reference
(`kernel_fn(grad_output, cos, sin) -> grad_x`, :126-170): the exact gradient
of the interleaved-pair forward, i.e. the rotation of grad_output by -theta on
the same pairs.  cos / sin are the forward's (N, D/2) tables.  (The reference's
backward assumes the rotate-half pairing with full-width (N, D) tables, which
is not the gradient of its own interleaved forward.)
"""
import torch

from kernels import _ak

KERNEL_TYPE = "rotary_embedding_backward"
BACKEND = "cuda_sm100a"


def kernel_fn(grad_output: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    assert grad_output.is_cuda
    return _ak.rope_bwd(grad_output, cos, sin)
