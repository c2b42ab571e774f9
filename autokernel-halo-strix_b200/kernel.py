"""Root-level facade re-exporting kernels.ce_fused (mirrors the reference's kernel.py:9-26)."""
from kernels.ce_fused import *  # noqa: F401,F403
from kernels.ce_fused import (  # noqa: F401
    BACKEND,
    BYTES_FN,
    FLOPS_FN,
    KERNEL_TYPE,
    MODEL_SHAPES,
    TEST_SIZES,
    TOLERANCES,
    _CrossEntropyHIP,
    _get_bwd_module,
    _get_fwd_module,
    ce_full,
    kernel_fn,
)
