"""ak_rmsnorm_bwd_noalloc: the RMSNorm backward for callers that cannot allocate
device memory (their host owns all of it, or their plugin ABI passes only
inputs and outputs).  Its scratch is a static device array inside the library,
so the check here is that, called through the C ABI twice in a row, it gives
the same dx and dw as the workspace-taking ak_rmsnorm_bwd within the fp32
tolerance used by every other test (the second call also shows that leftover
scratch contents from the first call do not leak into the result).

This file is named to be collected last."""
import ctypes

import pytest
import torch

from conftest import assert_fp32_close, assert_lowp_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,M,N", [(torch.float32, 8192, 768), (torch.bfloat16, 1000, 4096),
                                       (torch.float32, 37, 5000)])
def test_noalloc_matches_workspace_entry_point(dtype, M, N):
    from kernels import _ak
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, N, generator=g).to(dtype).cuda()
    w = (1 + 0.02 * torch.randn(N, generator=g)).to(dtype).cuda()
    for call in range(2):
        dy = torch.randn(M, N, generator=g).to(dtype).cuda()
        ref_dx, ref_dw = _ak.rmsnorm_bwd(x, w, dy, 1e-6)
        dx = torch.empty_like(x)
        dw = torch.empty(N, dtype=torch.float32, device="cuda")
        dt = _ak.dtype_code(x)
        _ak.call("ak_rmsnorm_bwd_noalloc", _ak.ptr(dx), _ak.ptr(dw), _ak.F32, _ak.ptr(dy), _ak.ptr(x), _ak.ptr(w),
                 M, N, ctypes.c_float(1e-6), dt, dt, _ak.stream(x.device))
        torch.cuda.synchronize()
        (assert_fp32_close if dtype == torch.float32 else assert_lowp_close)(dx, ref_dx, what=f"dx call {call}")
        assert_fp32_close(dw, ref_dw, what=f"dw call {call}")


def test_noalloc_rejects_too_wide_rows():
    from kernels import _ak
    N = (1 << 20) + 1
    x = torch.zeros(1, N, device="cuda")
    w = torch.ones(N, device="cuda")
    dw = torch.empty(N, device="cuda")
    with pytest.raises(_ak.AkError, match="exceeds the static scratch"):
        _ak.call("ak_rmsnorm_bwd_noalloc", _ak.ptr(x), _ak.ptr(dw), _ak.F32, _ak.ptr(x), _ak.ptr(x), _ak.ptr(w),
                 1, N, ctypes.c_float(1e-6), _ak.F32, _ak.F32, _ak.stream(x.device))
