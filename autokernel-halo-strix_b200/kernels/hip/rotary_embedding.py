"""Rotary position embedding (interleaved pairs) on B200.

Drop-in for kernels/hip/rotary_embedding.py of the reference: `kernel_fn(x,
cos, sin)` and `kernel_fn_fp32(x, cos, sin)` (:253-300) with the semantics of
reference.rotary_embedding_ref (reference.py:63-69).  x is (B, H, N, D); cos /
sin are (N, D/2) (or broadcastable (..., N, D/2)) and are used in fp32.  Both
entry points run the same kernel: fp32 arithmetic, one rounding to x's dtype
(the reference's fp16 `kernel_fn` rounds each product in fp16).  x may be a
strided view (e.g. heads of a fused QKV projection); the result is dense.
"""
import torch

from kernels import _ak

KERNEL_TYPE = "rotary_embedding"
BACKEND = "cuda_sm100a"


def kernel_fn(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    assert x.is_cuda
    return _ak.rope_fwd(x, cos, sin)


def kernel_fn_fp32(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    assert x.is_cuda
    return _ak.rope_fwd(x, cos, sin)
