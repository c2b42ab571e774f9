"""Row softmax (last dim) on B200, forward and backward.

Drop-in for kernels/hip/softmax.py (`kernel_fn`, softmax.py:339-360) with the
semantics of reference.softmax_ref (reference.py:15-17).  The reference has an
fp16-only forward kernel whose launcher leaves rows >= 65535 unwritten
(softmax.py:175-176, 293) and no backward; here every row of every dtype
(fp32/bf16/fp16) is computed, and `kernel_fn` is differentiable through the
`torch.ops.autokernel.softmax` custom op (backward dx = y * (dy - sum(dy*y))).
"""
import torch

KERNEL_TYPE = "softmax"
BACKEND = "cuda_sm100a"


def kernel_fn(x: torch.Tensor) -> torch.Tensor:
    """softmax(x, dim=-1) for a CUDA tensor of any rank."""
    assert x.is_cuda
    import kernels.hip._torch_ops  # noqa: F401  (registers the custom op)
    return torch.ops.autokernel.softmax(x)
