"""ctypes binding of libak_b200.so (the sm_100a kernels) plus tensor-level wrappers.

Every wrapper allocates its outputs and workspaces with PyTorch on the input's
device, passes raw pointers and PyTorch's current stream to the C ABI
(`include/ak_b200.h`), and raises `AkError` with the library's message when a
call fails.  There is no CPU or PyTorch fallback: inputs must be CUDA tensors
and the shared library must be present, otherwise the call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Optional, Sequence

import torch

LIB_PATH = Path(__file__).resolve().parent.parent / "libak_b200.so"

F32, BF16, F16 = 0, 1, 2
_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_vp, _i64, _f, _i, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_size_t

# name -> argtypes (all entry points return int status)
SIGNATURES = {
    "ak_version": [],
    "ak_rmsnorm_fwd": [_vp, _vp, _vp, _vp, _i64, _i64, _f, _i, _i, _vp],
    "ak_rmsnorm_bwd_workspace_size": [_i64, _i64, ctypes.POINTER(_sz)],
    "ak_rmsnorm_bwd": [_vp, _vp, _i, _vp, _sz, _vp, _vp, _vp, _i64, _i64, _f, _i, _i, _vp],
    "ak_rmsnorm_bwd_noalloc": [_vp, _vp, _i, _vp, _vp, _vp, _i64, _i64, _f, _i, _i, _vp],
    "ak_fused_res_rmsnorm_fwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _i, _i, _vp],
    "ak_fused_res_rmsnorm_bwd": [_vp, _vp, _i, _vp, _sz, _vp, _vp, _vp, _vp, _i64, _i64, _f, _i, _i, _vp],
    "ak_silu_gate_mul_fwd": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _vp],
    "ak_silu_gate_mul_bwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i, _vp],
    "ak_rope_fwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i, _vp],
    "ak_rope_bwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i, _vp],
    "ak_rope_strided": [_vp, _vp, _vp, _vp] + [_i64] * 10 + [_i, _i, _vp],
    "ak_scale_by_device_scalar": [_vp, _i64, _vp, _i, _vp],
    "ak_transpose": [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i, _vp],
    "ak_rmsnorm_fwd_mixed": [_vp, _i, _vp, _i, _vp, _i, _i64, _i64, _f, _vp],
    "ak_fused_res_rmsnorm_fwd_mixed": [_vp, _vp, _i, _vp, _i, _vp, _i, _vp, _i, _i64, _i64, _f, _vp],
    "ak_rmsnorm_bwd_mixed": [_vp, _vp, _vp, _i, _vp, _sz, _vp, _vp, _i, _vp, _i, _vp, _i, _i64, _i64, _f, _vp],
    "ak_softmax_fwd": [_vp, _vp, _i64, _i64, _i, _vp],
    "ak_softmax_bwd": [_vp, _vp, _vp, _i64, _i64, _i, _vp],
    "ak_ce_rows_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _i64, _f, _f, _vp, _i, _vp],
    "ak_ce_rows_bwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _i64, _f, _f, _vp, _f, _i, _vp],
    "ak_ce_rows_reduce": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _vp],
    "ak_ce_inv_valid": [_vp, _vp, _i64, _i64, _vp],
    "ak_linear_ce_logits_grad_workspace_size": [_i64, _i64, ctypes.POINTER(_sz)],
    "ak_linear_ce_logits_grad": [_vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _vp, _vp],
    "ak_linear_ce_workspace_size": [_i64, _i64, _i64, ctypes.POINTER(_sz)],
    "ak_linear_ce_fwdbwd": [_vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _vp,
                            _vp],
    "ak_scan1_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ak_scan1_bwd_workspace_size": [_i64, _i64, _i64, ctypes.POINTER(_sz)],
    "ak_scan1_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ak_scan1_carries_size": [_i64, _i64, _i64, ctypes.POINTER(_sz)],
    "ak_scan1_fwd_ex": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ak_scan1_bwd_ex": [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ak_causal_conv1d_fwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _i, _vp],
    "ak_causal_conv1d_bwd_workspace_size": [_i64, _i64, _i64, _i64, ctypes.POINTER(_sz)],
    "ak_causal_conv1d_bwd": [_vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i, _i, _vp],
    "ak_selective_scan_state_stride": [],
    "ak_selective_scan_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                              _i64, _i64, _i64, _i64, _i64, _i, _vp, _vp],
    "ak_selective_scan_bwd_workspace_size": [_i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_sz)],
    "ak_selective_scan_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp,
                              _vp, _vp, _vp, _vp, _i, _i64, _i64, _i64, _i64, _i64, _i, _vp, _vp],
    "ak_tc_gemm": [_vp, _i, _vp, _vp, _i64, _i64, _i64, _i, _i, _i, _vp, _vp],
    "ak_status_device_pointer": [_vp, ctypes.POINTER(_vp)],
    "ak_test_bounded_wait": [_vp, _i, _vp],
}


class AkError(RuntimeError):
    """A libak_b200 entry point returned a nonzero status."""


_lib: Optional[ctypes.CDLL] = None
_lock = threading.RLock()  # reentrant: the status words are set up through call() under it


def lib() -> ctypes.CDLL:
    """Load libak_b200.so once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise ImportError(
                        f"libak_b200.so not found at {LIB_PATH}; build it with "
                        "`python autokernel-halo-strix_b200/csrc/build.py`")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, argtypes in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = argtypes
                    fn.restype = ctypes.c_int
                handle.ak_last_error.argtypes = []
                handle.ak_last_error.restype = ctypes.c_char_p
                _lib = handle
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().ak_last_error().decode(errors="replace")
        raise AkError(f"{name} failed (status {rc}): {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("autokernel B200 kernels need CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    if dev is None:
        raise RuntimeError("no tensor given")
    return dev


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _size_query(name: str, *dims: int) -> int:
    out = ctypes.c_size_t(0)
    call(name, *dims, ctypes.byref(out))
    return int(out.value)


# ---------------------------------------------------------------------------
# Device status words (bounded-wait timeouts)
# ---------------------------------------------------------------------------
AK_ERR_TIMEOUT = 5
STATUS_SLOTS = ("selective_scan_fwd", "selective_scan_bwd", "linear_ce", "bounded_wait_test")


class _StatusWords:
    """One pinned host int32 per kernel family on one device.  The kernels write AK_ERR_TIMEOUT
    into it through its device address when a bounded wait runs out, so the host reads a failure
    without a CUDA call: the next call of the same family raises it, and `check_status` raises it
    after synchronising."""

    def __init__(self, device: torch.device):
        self.host = torch.zeros(len(STATUS_SLOTS), dtype=torch.int32, pin_memory=True)
        dev_ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            call("ak_status_device_pointer", ctypes.c_void_p(self.host.data_ptr()), ctypes.byref(dev_ptr))
        self.base = int(dev_ptr.value)

    def raise_if_set(self, slots) -> None:
        for i in slots:
            code = int(self.host[i])
            if code != 0:
                self.host[i] = 0
                raise AkError(f"{STATUS_SLOTS[i]}: a bounded device-side wait gave up (status {code}, "
                              "AK_ERR_TIMEOUT); the outputs of that call are invalid")


_status: dict = {}


def _status_words(device: torch.device) -> _StatusWords:
    key = device.index if device.index is not None else torch.cuda.current_device()
    sw = _status.get(key)
    if sw is None:
        with _lock:
            sw = _status.get(key)
            if sw is None:
                sw = _status[key] = _StatusWords(torch.device("cuda", key))
    return sw


def status_ptr(device: torch.device, slot: str):
    """Device address of the status word of `slot`; raises first if an earlier call of that
    family reported a timeout."""
    sw = _status_words(device)
    i = STATUS_SLOTS.index(slot)
    sw.raise_if_set((i,))
    return ctypes.c_void_p(sw.base + 4 * i)


def check_status(device: Optional[torch.device] = None, synchronize: bool = True) -> None:
    """Raise AkError if any kernel on `device` (default: current) reported a bounded-wait
    timeout; with synchronize=True every call issued so far is covered."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if synchronize:
        torch.cuda.synchronize(dev)
    _status_words(dev).raise_if_set(range(len(STATUS_SLOTS)))


def test_bounded_wait(device: torch.device, max_spins: int = 1000) -> None:
    """Run the library's bounded-wait probe (a wait nothing completes), then check the status."""
    dev = torch.device(device)
    call("ak_test_bounded_wait", status_ptr(dev, "bounded_wait_test"), int(max_spins), stream(dev))
    check_status(dev, synchronize=True)


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------
def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, want_rstd: bool = False):
    dev = require_cuda(x, w)
    x = x.contiguous()
    w = w.contiguous()
    N = x.shape[-1]
    M = x.numel() // N if N else 0
    y = torch.empty_like(x)
    rstd = torch.empty(M, dtype=torch.float32, device=dev) if want_rstd else None
    call("ak_rmsnorm_fwd", ptr(y), ptr(rstd), ptr(x), ptr(w), M, N, float(eps), dtype_code(x), dtype_code(w),
         stream(dev))
    return (y, rstd) if want_rstd else y


def rmsnorm_bwd(x: torch.Tensor, w: torch.Tensor, dy: torch.Tensor, eps: float = 1e-6,
                dw_dtype: torch.dtype = torch.float32):
    dev = require_cuda(x, w, dy)
    x = x.contiguous()
    w = w.contiguous()
    dy = dy.to(x.dtype).contiguous()
    N = x.shape[-1]
    M = x.numel() // N if N else 0
    dx = torch.empty_like(x)
    dw = torch.empty(N, dtype=dw_dtype, device=dev)
    ws_bytes = _size_query("ak_rmsnorm_bwd_workspace_size", M, N)
    ws = workspace(ws_bytes, dev)
    call("ak_rmsnorm_bwd", ptr(dx), ptr(dw), _DT[dw_dtype], ptr(ws), ws_bytes, ptr(dy), ptr(x), ptr(w), M, N,
         float(eps), dtype_code(x), dtype_code(w), stream(dev))
    return dx, dw


# ---------------------------------------------------------------------------
# Fused residual add + RMSNorm
# ---------------------------------------------------------------------------
def fused_res_rmsnorm_fwd(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float = 1e-6,
                          want_hidden: bool = True):
    """Returns (hidden or None, normed), both shaped and typed like x."""
    dev = require_cuda(x, residual, w)
    if residual.shape != x.shape:
        raise ValueError(f"fused_res_rmsnorm: residual {tuple(residual.shape)} != x {tuple(x.shape)}")
    x = x.contiguous()
    residual = residual.to(x.dtype).contiguous()
    w = w.contiguous()
    N = x.shape[-1]
    M = x.numel() // N if N else 0
    normed = torch.empty_like(x)
    hidden = torch.empty_like(x) if want_hidden else None
    call("ak_fused_res_rmsnorm_fwd", ptr(hidden), ptr(normed), ptr(x), ptr(residual), ptr(w), M, N, float(eps),
         dtype_code(x), dtype_code(w), stream(dev))
    return hidden, normed


def fused_res_rmsnorm_bwd(hidden: torch.Tensor, w: torch.Tensor, grad_hidden: Optional[torch.Tensor],
                          grad_normed: torch.Tensor, eps: float = 1e-6, dw_dtype: Optional[torch.dtype] = None):
    """Returns (dx, dw); dx is also the residual's gradient. dw defaults to fp32."""
    dev = require_cuda(hidden, w, grad_hidden, grad_normed)
    dw_dtype = dw_dtype or torch.float32
    hidden = hidden.contiguous()
    w = w.contiguous()
    gn = grad_normed.to(hidden.dtype).contiguous()
    gh = grad_hidden.to(hidden.dtype).contiguous() if grad_hidden is not None else None
    N = hidden.shape[-1]
    M = hidden.numel() // N if N else 0
    dx = torch.empty_like(hidden)
    dw = torch.empty(N, dtype=dw_dtype, device=dev)
    ws_bytes = _size_query("ak_rmsnorm_bwd_workspace_size", M, N)
    ws = workspace(ws_bytes, dev)
    call("ak_fused_res_rmsnorm_bwd", ptr(dx), ptr(dw), _DT[dw_dtype], ptr(ws), ws_bytes, ptr(gh), ptr(gn),
         ptr(hidden), ptr(w), M, N, float(eps), dtype_code(hidden), dtype_code(w), stream(dev))
    return dx, dw


# ---------------------------------------------------------------------------
# Mixed-precision RMSNorm: fp32 residual stream, 16-bit autocast activations
# ---------------------------------------------------------------------------
def rmsnorm_fwd_mixed(x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
    """y = rmsnorm(x fp32) * w written in `out_dtype` (one rounding)."""
    dev = require_cuda(x, w)
    x, w = x.contiguous(), w.contiguous()
    N = x.shape[-1]
    M = x.numel() // N if N else 0
    y = torch.empty(x.shape, dtype=out_dtype, device=dev)
    call("ak_rmsnorm_fwd_mixed", ptr(y), _DT[out_dtype], ptr(x), dtype_code(x), ptr(w), dtype_code(w), M, N,
         float(eps), stream(dev))
    return y


def fused_res_rmsnorm_fwd_mixed(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """hidden (residual's dtype, fp32) = x (16-bit) + residual; normed (x's dtype) = rmsnorm(hidden) * w."""
    dev = require_cuda(x, residual, w)
    x, residual, w = x.contiguous(), residual.contiguous(), w.contiguous()
    N = x.shape[-1]
    M = x.numel() // N if N else 0
    hidden = torch.empty(x.shape, dtype=residual.dtype, device=dev)
    normed = torch.empty_like(x)
    call("ak_fused_res_rmsnorm_fwd_mixed", ptr(hidden), ptr(normed), dtype_code(normed), ptr(x), dtype_code(x),
         ptr(residual), dtype_code(residual), ptr(w), dtype_code(w), M, N, float(eps), stream(dev))
    return hidden, normed


def rmsnorm_bwd_mixed(x: torch.Tensor, w: torch.Tensor, dy: torch.Tensor, eps: float,
                      grad_hidden: Optional[torch.Tensor] = None, want_lo: bool = False):
    """x fp32, dy 16-bit.  Returns (dx fp32, dx in dy's dtype or None, dw fp32)."""
    dev = require_cuda(x, w, dy, grad_hidden)
    x, w, dy = x.contiguous(), w.contiguous(), dy.contiguous()
    gh = grad_hidden.to(x.dtype).contiguous() if grad_hidden is not None else None
    N = x.shape[-1]
    M = x.numel() // N if N else 0
    dx = torch.empty_like(x)
    dx2 = torch.empty_like(dy) if want_lo else None
    dw = torch.empty(N, dtype=torch.float32, device=dev)
    ws_bytes = _size_query("ak_rmsnorm_bwd_workspace_size", M, N)
    ws = workspace(ws_bytes, dev)
    call("ak_rmsnorm_bwd_mixed", ptr(dx), ptr(dx2), ptr(dw), F32, ptr(ws), ws_bytes, ptr(gh), ptr(dy),
         dtype_code(dy), ptr(x), dtype_code(x), ptr(w), dtype_code(w), M, N, float(eps), stream(dev))
    return dx, dx2, dw


# ---------------------------------------------------------------------------
# SiLU gate multiply (SwiGLU body)
# ---------------------------------------------------------------------------
def _rows(t: torch.Tensor, cols: int) -> torch.Tensor:
    """(rows, cols) view with unit column stride (a copy only when no such view exists)."""
    if t.stride(-1) == 1:
        try:
            v = t.view(-1, cols)
            if v.stride(1) == 1:
                return v
        except RuntimeError:
            pass
    return t.contiguous().view(-1, cols)


def silu_gate_mul_fwd(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up; gate / up may be strided row views (e.g. halves of one packed tensor)."""
    dev = require_cuda(gate, up)
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError(f"silu_gate_mul: gate {tuple(gate.shape)}/{gate.dtype} vs up {tuple(up.shape)}/{up.dtype}")
    cols = gate.shape[-1]
    y = torch.empty(gate.shape, dtype=gate.dtype, device=dev)
    if gate.numel() == 0:
        return y
    g2, u2 = _rows(gate, cols), _rows(up, cols)
    call("ak_silu_gate_mul_fwd", ptr(y), ptr(g2), ptr(u2), g2.shape[0], cols, g2.stride(0), u2.stride(0),
         dtype_code(gate), stream(dev))
    return y


def silu_gate_mul_bwd(gate: torch.Tensor, up: torch.Tensor, dy: torch.Tensor,
                      packed_out: Optional[torch.Tensor] = None):
    """Returns (d gate, d up).  With `packed_out` ((..., 2*cols), contiguous) both are
    written into its two halves and returned as views of it."""
    dev = require_cuda(gate, up, dy)
    cols = gate.shape[-1]
    if packed_out is not None:
        if packed_out.shape[-1] != 2 * cols or not packed_out.is_contiguous():
            raise ValueError("silu_gate_mul_bwd: packed_out must be contiguous (..., 2*cols)")
        dg, du = packed_out[..., :cols], packed_out[..., cols:]
    else:
        dg, du = torch.empty(gate.shape, dtype=gate.dtype, device=dev), torch.empty(gate.shape, dtype=gate.dtype,
                                                                                     device=dev)
    if gate.numel() == 0:
        return dg, du
    g2, u2 = _rows(gate, cols), _rows(up, cols)
    y2 = _rows(dy.to(gate.dtype), cols)
    if y2.stride(0) != cols:
        y2 = y2.contiguous()
    dg2, du2 = dg.view(-1, cols) if packed_out is None else packed_out.view(-1, 2 * cols)[:, :cols], \
        du.view(-1, cols) if packed_out is None else packed_out.view(-1, 2 * cols)[:, cols:]
    call("ak_silu_gate_mul_bwd", ptr(dg2), ptr(du2), ptr(g2), ptr(u2), ptr(y2), g2.shape[0], cols, g2.stride(0),
         u2.stride(0), dg2.stride(0), du2.stride(0), dtype_code(gate), stream(dev))
    return dg, du


# ---------------------------------------------------------------------------
# Rotary position embedding (interleaved pairs), x (B, H, N, D)
# ---------------------------------------------------------------------------
def _rope_tables(t: torch.Tensor, N: int, D: int) -> torch.Tensor:
    """fp32 (N, D/2) table from any (..., N', D/2) broadcast form with N' >= N."""
    if t.shape[-1] != D // 2:
        raise ValueError(f"rotary: tables must have last dim D/2 = {D // 2} (interleaved pairs), got {t.shape[-1]}")
    t2 = t.detach().float().reshape(-1, D // 2) if t.dim() != 2 else t.float()
    if t2.shape[0] < N:
        raise ValueError(f"rotary: table has {t2.shape[0]} positions < sequence length {N}")
    return t2[:N].contiguous()


def _rope(name: str, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    dev = require_cuda(x, cos, sin)
    if x.dim() != 4:
        raise ValueError(f"rotary: x must be (B, H, N, D), got {tuple(x.shape)}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    B, H, N, D = x.shape
    c, s = _rope_tables(cos, N, D), _rope_tables(sin, N, D)
    y = torch.empty((B, H, N, D), dtype=x.dtype, device=dev)
    if x.numel():
        call(name, ptr(y), ptr(x), ptr(c), ptr(s), B, H, N, D, x.stride(0), x.stride(1), x.stride(2), dtype_code(x),
             stream(dev))
    return y


def rope_fwd(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs of x (B, H, N, D; any strides with unit D stride) -> dense (B, H, N, D)."""
    return _rope("ak_rope_fwd", x, cos, sin)


def rope_bwd(dy: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return _rope("ak_rope_bwd", dy, cos, sin)


def scale_by_device_scalar_(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """In place x *= scale (a one-element tensor read on the device; nothing is written when it
    is exactly 1).  No host sync."""
    dev = require_cuda(x, scale)
    if not x.is_contiguous():
        raise ValueError("scale_by_device_scalar_: x must be contiguous")
    s = scale.reshape(1).to(torch.float32)
    if x.numel():
        call("ak_scale_by_device_scalar", ptr(x), x.numel(), ptr(s), dtype_code(x), stream(dev))
    return x


def rope_into(y: torch.Tensor, x: torch.Tensor, cos, sin, mode: int) -> torch.Tensor:
    """y <- rotation of x (mode 1), its inverse (mode -1) or a copy (mode 0); x and y are
    (B, H, N, D) views with any strides and unit stride along D (e.g. head slices of packed
    (B, N, W) projections or gradients).  cos / sin: (N, D/2) fp32, unused for mode 0."""
    dev = require_cuda(x, y)
    if x.dim() != 4 or y.shape != x.shape or y.dtype != x.dtype:
        raise ValueError(f"rope_into: x {tuple(x.shape)} {x.dtype} -> y {tuple(y.shape)} {y.dtype}")
    if y.stride(-1) != 1:
        raise ValueError("rope_into: y needs unit stride along D")
    if x.stride(-1) != 1:
        x = x.contiguous()
    B, H, N, D = x.shape
    if mode not in (1, -1, 0):
        raise ValueError(f"rope_into: mode must be 1, -1 or 0, got {mode}")
    c = s = None
    if mode != 0:
        c, s = _rope_tables(cos, N, D), _rope_tables(sin, N, D)
    if x.numel():
        call("ak_rope_strided", ptr(y), ptr(x), ptr(c), ptr(s), B, H, N, D, x.stride(0), x.stride(1), x.stride(2), y.stride(0),
             y.stride(1), y.stride(2), mode, dtype_code(x), stream(dev))
    return y


# ---------------------------------------------------------------------------
# Batched last-two-dims transpose
# ---------------------------------------------------------------------------
def transpose_into(out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """out[b, c, r] = x[b, r, c] for 3-D x (B, R, C) and out (B, C, R); both may be strided
    views as long as their last dimension has unit stride."""
    dev = require_cuda(x, out)
    if x.dim() != 3 or out.shape != (x.shape[0], x.shape[2], x.shape[1]) or x.dtype != out.dtype:
        raise ValueError(f"transpose: x {tuple(x.shape)} -> out {tuple(out.shape)}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out.stride(-1) != 1:
        raise ValueError("transpose: out needs unit stride along its last dimension")
    B, R, C = x.shape
    if x.numel():
        call("ak_transpose", ptr(out), ptr(x), B, R, C, x.stride(0), x.stride(1), out.stride(0), out.stride(1),
             dtype_code(x), stream(dev))
    return out


def transpose_bt(x: torch.Tensor) -> torch.Tensor:
    """Contiguous x.transpose(-1, -2) of a 3-D tensor (B, R, C) -> (B, C, R)."""
    out = torch.empty((x.shape[0], x.shape[2], x.shape[1]), dtype=x.dtype, device=x.device)
    return transpose_into(out, x)


# ---------------------------------------------------------------------------
# Softmax (last dim)
# ---------------------------------------------------------------------------
def softmax_fwd(x: torch.Tensor) -> torch.Tensor:
    dev = require_cuda(x)
    x = x.contiguous()
    cols = x.shape[-1] if x.dim() > 0 else 1
    rows = x.numel() // cols if cols else 0
    y = torch.empty_like(x)
    if x.numel():
        call("ak_softmax_fwd", ptr(y), ptr(x), rows, cols, dtype_code(x), stream(dev))
    return y


def softmax_bwd(y: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    dev = require_cuda(y, dy)
    y = y.contiguous()
    dy = dy.to(y.dtype).contiguous()
    cols = y.shape[-1] if y.dim() > 0 else 1
    rows = y.numel() // cols if cols else 0
    dx = torch.empty_like(y)
    if y.numel():
        call("ak_softmax_bwd", ptr(dx), ptr(y), ptr(dy), rows, cols, dtype_code(y), stream(dev))
    return dx


# ---------------------------------------------------------------------------
# Cross entropy over logit rows
# ---------------------------------------------------------------------------
def ce_rows_fwd(logits: torch.Tensor, targets: torch.Tensor, softcap: float = 0.0, ignore_index: int = -100,
                label_smoothing: float = 0.0, write_grad: bool = False, save_max_sum: bool = False,
                scale_grad: float = 1.0, scale_dev: Optional[torch.Tensor] = None):
    """Returns [losses, lse, row_max, row_sum, grad] (absent ones are None)."""
    dev = require_cuda(logits, targets)
    logits = logits.contiguous()
    targets = targets.to(torch.int64).contiguous()
    B, V = logits.shape
    f32 = dict(dtype=torch.float32, device=dev)
    losses = torch.empty(B, **f32)
    lse = torch.empty(B, **f32)
    rmax = torch.empty(B, **f32) if save_max_sum else None
    rsum = torch.empty(B, **f32) if save_max_sum else None
    grad = torch.empty_like(logits) if write_grad else None
    if scale_dev is not None:
        scale_dev = scale_dev.to(torch.float32).contiguous()
    call("ak_ce_rows_fwd", ptr(losses), ptr(lse), ptr(rmax), ptr(rsum), ptr(grad), ptr(logits), ptr(targets), B, V,
         float(softcap), int(ignore_index), float(label_smoothing), float(scale_grad), ptr(scale_dev),
         dtype_code(logits), stream(dev))
    return [losses, lse, rmax, rsum, grad]


def ce_rows_bwd(logits, targets, row_max, row_sum, softcap=0.0, ignore_index=-100, label_smoothing=0.0,
                scale=1.0, scale_dev: Optional[torch.Tensor] = None, z_coef: float = 0.0,
                out: Optional[torch.Tensor] = None):
    dev = require_cuda(logits, targets, row_max, row_sum)
    logits = logits.contiguous()
    targets = targets.to(torch.int64).contiguous()
    B, V = logits.shape
    grad = torch.empty_like(logits) if out is None else out
    if scale_dev is not None:
        scale_dev = scale_dev.to(torch.float32).contiguous()
    call("ak_ce_rows_bwd", ptr(grad), ptr(logits), ptr(targets), ptr(row_max.contiguous()),
         ptr(row_sum.contiguous()), B, V, float(softcap), int(ignore_index), float(label_smoothing), float(scale),
         ptr(scale_dev), float(z_coef), dtype_code(logits), stream(dev))
    return grad


def ce_rows_reduce(losses, lse, targets, ignore_index=-100, z_loss_weight=0.0):
    """Device-side mean over valid rows; returns (loss 0-d fp32, n_valid 0-d fp32)."""
    dev = require_cuda(losses, targets)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    nvalid = torch.empty((), dtype=torch.float32, device=dev)
    targets = targets.to(torch.int64).contiguous()
    call("ak_ce_rows_reduce", ptr(loss), ptr(nvalid), ptr(losses.contiguous()),
         ptr(lse.contiguous() if lse is not None else None), ptr(targets), targets.numel(), int(ignore_index),
         float(z_loss_weight), stream(dev))
    return loss, nvalid


def ce_inv_valid(targets: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    dev = require_cuda(targets)
    targets = targets.to(torch.int64).contiguous()
    inv = torch.empty((), dtype=torch.float32, device=dev)
    call("ak_ce_inv_valid", ptr(inv), ptr(targets), targets.numel(), int(ignore_index), stream(dev))
    return inv


def linear_ce_supported(hidden: torch.Tensor, weight: torch.Tensor) -> bool:
    N, D = hidden.shape
    V = weight.shape[0]
    return (hidden.dtype in (torch.bfloat16, torch.float16) and weight.dtype == hidden.dtype
            and N % 8 == 0 and D % 8 == 0 and V % 8 == 0 and N > 0)


def linear_ce_logits_grad(hidden, weight, labels, ignore_index=-100):
    """tcgen05 logits GEMM with fused softmax statistics, then G = dloss/dlogits in place.
    Returns (loss 0-d fp32, lse [N] fp32, G [N, V] in hidden's dtype)."""
    dev = require_cuda(hidden, weight, labels)
    h = hidden.contiguous()
    w = weight.contiguous()
    lab = labels.to(torch.int64).contiguous()
    N, D = h.shape
    V = w.shape[0]
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    G = torch.empty(N, V, dtype=h.dtype, device=dev)
    ws_bytes = _size_query("ak_linear_ce_logits_grad_workspace_size", N, V)
    ws = workspace(ws_bytes, dev)
    call("ak_linear_ce_logits_grad", ptr(loss), ptr(lse), ptr(G), ptr(ws), ws_bytes, ptr(h), ptr(w), ptr(lab), N, D,
         V, int(ignore_index), dtype_code(h), status_ptr(dev, "linear_ce"), stream(dev))
    return loss, lse, G


def linear_ce_fwdbwd(hidden, weight, labels, ignore_index=-100, need_dh=True, need_dw=True,
                     inv_valid: Optional[torch.Tensor] = None):
    """Fused tcgen05 linear + CE: returns (loss 0-d fp32, lse [N] fp32, dH or None, dW or None).

    inv_valid (optional one-element fp32 CUDA tensor): 1 / n_valid to use instead of this call's
    own count; with the count of all shards, loss and dW are this shard's parts of their sums."""
    dev = require_cuda(hidden, weight, labels)
    h = hidden.contiguous()
    w = weight.contiguous()
    lab = labels.to(torch.int64).contiguous()
    N, D = h.shape
    V = w.shape[0]
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    dH = torch.empty_like(h) if need_dh else None
    dW = torch.empty_like(w) if need_dw else None
    ws_bytes = _size_query("ak_linear_ce_workspace_size", N, D, V)
    ws = workspace(ws_bytes, dev)
    if inv_valid is not None:
        inv_valid = inv_valid.reshape(1).to(torch.float32).contiguous()
    call("ak_linear_ce_fwdbwd", ptr(loss), ptr(lse), ptr(dH), ptr(dW), ptr(ws), ws_bytes, ptr(h), ptr(w), ptr(lab),
         ptr(inv_valid), N, D, V, int(ignore_index), dtype_code(h), status_ptr(dev, "linear_ce"), stream(dev))
    return loss, lse, dH, dW


def tc_gemm(a: torch.Tensor, b: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """a @ b on the library's tcgen05 GEMM for 2-D bf16 / fp16 a (M, K) and b (K, N).  Either
    operand may be a plain tensor or the transpose view of one (its K or its M / N dimension
    contiguous); nothing is copied.  Returns a dense (M, N) tensor in out_dtype (default a's)."""
    dev = require_cuda(a, b)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0] or a.dtype != b.dtype:
        raise ValueError(f"tc_gemm: {tuple(a.shape)} {a.dtype} @ {tuple(b.shape)} {b.dtype}")
    M, K = a.shape
    N = b.shape[1]
    # A[M][K] K-contiguous (a_mn 0) or stored [K][M] (a_mn 1); B as N x K likewise; dense only
    if a.stride() == (K, 1):
        a_mn = 0
    elif a.stride() == (1, M):
        a_mn = 1
    else:
        a, a_mn = a.contiguous(), 0
    if b.stride() == (1, K):
        b_mn = 0  # b (K, N) is the transpose of a dense B[N][K]
    elif b.stride() == (N, 1):
        b_mn = 1
    else:
        b, b_mn = b.contiguous(), 1
    out_dtype = out_dtype or a.dtype
    c = torch.empty(M, N, dtype=out_dtype, device=dev)
    call("ak_tc_gemm", ptr(c), dtype_code(c), ptr(a), ptr(b), M, N, K, a_mn, b_mn, dtype_code(a),
         status_ptr(dev, "linear_ce"), stream(dev))
    return c


# ---------------------------------------------------------------------------
# Collapsed selective scan (fp32, (B, L, d))
# ---------------------------------------------------------------------------
def _f32c(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.float32:
        raise TypeError(f"collapsed selective scan is fp32-only (got {t.dtype})")
    return t.contiguous()


def scan1_fwd(dA, dBx, C, D, x, save_carries: bool = False):
    """y (and, with save_carries, the chunk-start states the backward needs)."""
    dev = require_cuda(dA, dBx, C, D, x)
    dA, dBx, C, D, x = map(_f32c, (dA, dBx, C, D, x))
    if dA.dim() != 3:
        raise ValueError("dA must be 3D [batch, seq, d_inner]")
    B, L, d = dA.shape
    y = torch.empty_like(dA)
    carries = None
    if save_carries:
        nbytes = _size_query("ak_scan1_carries_size", B, L, d)
        carries = torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=dev)
    call("ak_scan1_fwd_ex", ptr(y), ptr(carries), ptr(dA), ptr(dBx), ptr(C), ptr(D), ptr(x), B, L, d, stream(dev))
    return (y, carries) if save_carries else y


def scan1_bwd(dA, dBx, C, D, x, gy, carries=None):
    """(gdA, gdBx, gC, gD, gx); `carries` from scan1_fwd(save_carries=True) skips the pass that
    re-derives the chunk-start states."""
    dev = require_cuda(dA, dBx, C, D, x, gy)
    dA, dBx, C, D, x, gy = map(_f32c, (dA, dBx, C, D, x, gy))
    B, L, d = dA.shape
    gdA, gdBx, gC, gx = (torch.empty_like(dA) for _ in range(4))
    gD = torch.empty(d, dtype=torch.float32, device=dev)
    if carries is not None:
        need = _size_query("ak_scan1_carries_size", B, L, d)
        if carries.dtype != torch.float32 or not carries.is_contiguous() or carries.numel() * 4 < need:
            raise ValueError("scan1_bwd: carries do not match this shape (use scan1_fwd(save_carries=True))")
        ws_bytes = max(B * d * 4, 4)
    else:
        ws_bytes = _size_query("ak_scan1_bwd_workspace_size", B, L, d)
    ws = workspace(ws_bytes, dev)
    call("ak_scan1_bwd_ex", ptr(gdA), ptr(gdBx), ptr(gC), ptr(gD), ptr(gx), ptr(ws), ws_bytes, ptr(carries),
         ptr(dA), ptr(dBx), ptr(C), ptr(D), ptr(x), ptr(gy), B, L, d, stream(dev))
    return gdA, gdBx, gC, gD, gx


# ---------------------------------------------------------------------------
# Mamba-style selective scan ((batch, dim, L), N states)
# ---------------------------------------------------------------------------
def state_stride() -> int:
    return int(lib().ak_selective_scan_state_stride())


def _bc4(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 3:
        return t.unsqueeze(1)
    if t.dim() == 4:
        return t
    raise NotImplementedError("only input-dependent B/C of shape (batch, N, L) or (batch, G, N, L) are supported")


def selective_scan_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                       save_states: bool = True):
    """Returns (out, last_state, chunk_states)."""
    dev = require_cuda(u, delta, A, B, C, D, z, delta_bias)
    if A.is_complex():
        raise NotImplementedError("complex A is not supported")
    u = u.contiguous()
    dtype = u.dtype
    delta = delta.to(dtype).contiguous()
    B4 = _bc4(B).to(dtype).contiguous()
    C4 = _bc4(C).to(dtype).contiguous()
    if B4.shape[1] != C4.shape[1]:
        raise ValueError("B and C must have the same number of groups")
    A = A.to(torch.float32).contiguous()
    D = D.to(torch.float32).contiguous() if D is not None else None
    z = z.to(dtype).contiguous() if z is not None else None
    delta_bias = delta_bias.to(torch.float32).contiguous() if delta_bias is not None else None
    batch, dim, L = u.shape
    N = A.shape[1]
    G = B4.shape[1]
    out = torch.empty_like(u)
    f32 = dict(dtype=torch.float32, device=dev)
    last = torch.empty(batch, dim, N, **f32)
    nsaved = (L + state_stride() - 1) // state_stride()
    states = torch.empty(batch, dim, nsaved, N, **f32) if save_states else None
    call("ak_selective_scan_fwd", ptr(out), ptr(last), ptr(states), ptr(u), ptr(delta), ptr(A), ptr(B4), ptr(C4),
         ptr(D), ptr(z), ptr(delta_bias), int(bool(delta_softplus)), batch, dim, L, N, G, dtype_code(u),
         status_ptr(dev, "selective_scan_fwd"), stream(dev))
    return out, last, states


def selective_scan_bwd(dout, u, delta, A, B, C, D, z, delta_bias, delta_softplus, chunk_states):
    """Returns (du, ddelta, dA, dB, dC, dD, dz, ddelta_bias) with B/C grads shaped like B/C."""
    dev = require_cuda(dout, u, delta, A, B, C)
    u = u.contiguous()
    dtype = u.dtype
    delta = delta.to(dtype).contiguous()
    dout = dout.to(dtype).contiguous()
    B4 = _bc4(B).to(dtype).contiguous()
    C4 = _bc4(C).to(dtype).contiguous()
    A = A.to(torch.float32).contiguous()
    D = D.to(torch.float32).contiguous() if D is not None else None
    z = z.to(dtype).contiguous() if z is not None else None
    delta_bias = delta_bias.to(torch.float32).contiguous() if delta_bias is not None else None
    batch, dim, L = u.shape
    N = A.shape[1]
    G = B4.shape[1]
    f32 = dict(dtype=torch.float32, device=dev)
    du = torch.empty_like(u)
    ddelta = torch.empty_like(u)
    dA = torch.empty(dim, N, **f32)
    dB = torch.empty_like(B4)
    dC = torch.empty_like(C4)
    dD = torch.empty(dim, **f32) if D is not None else None
    dz = torch.empty_like(u) if z is not None else None
    dbias = torch.empty(dim, **f32) if delta_bias is not None else None
    ws_bytes = _size_query("ak_selective_scan_bwd_workspace_size", batch, dim, L, N, G)
    ws = workspace(ws_bytes, dev)
    call("ak_selective_scan_bwd", ptr(du), ptr(ddelta), ptr(dA), ptr(dB), ptr(dC), ptr(dD), ptr(dz), ptr(dbias),
         ptr(ws), ws_bytes, ptr(dout), ptr(u), ptr(delta), ptr(A), ptr(B4), ptr(C4), ptr(D), ptr(z),
         ptr(delta_bias), ptr(chunk_states), int(bool(delta_softplus)), batch, dim, L, N, G, dtype_code(u),
         status_ptr(dev, "selective_scan_bwd"), stream(dev))
    if B.dim() == 3:
        dB = dB.squeeze(1)
    if C.dim() == 3:
        dC = dC.squeeze(1)
    return du, ddelta, dA, dB, dC, dD, dz, dbias


# ---------------------------------------------------------------------------
# Depthwise causal conv1d (B, D, T)
# ---------------------------------------------------------------------------
def causal_conv1d_fwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                      silu: bool = False) -> torch.Tensor:
    dev = require_cuda(x, weight, bias)
    if x.dim() != 3 or weight.dim() != 2 or weight.shape[0] != x.shape[1]:
        raise ValueError(f"causal_conv1d: x {tuple(x.shape)} / weight {tuple(weight.shape)} mismatch")
    x = x.contiguous()
    B, D, T = x.shape
    K = weight.shape[1]
    w32 = weight.float().contiguous()
    b32 = bias.float().contiguous() if bias is not None else None
    y = torch.empty_like(x)
    call("ak_causal_conv1d_fwd", ptr(y), ptr(x), ptr(w32), ptr(b32), B, D, T, K, int(bool(silu)), dtype_code(x), stream(dev))
    return y


def causal_conv1d_bwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], dy: torch.Tensor,
                      silu: bool = False):
    """Returns (dx, dweight fp32 (D, K), dbias fp32 (D) or None)."""
    dev = require_cuda(x, weight, bias, dy)
    x = x.contiguous()
    dy = dy.to(x.dtype).contiguous()
    B, D, T = x.shape
    K = weight.shape[1]
    w32 = weight.float().contiguous()
    b32 = bias.float().contiguous() if bias is not None else None
    dx = torch.empty_like(x)
    dw = torch.empty(D, K, dtype=torch.float32, device=dev)
    db = torch.empty(D, dtype=torch.float32, device=dev) if bias is not None else None
    ws_bytes = _size_query("ak_causal_conv1d_bwd_workspace_size", B, D, T, K)
    ws = workspace(ws_bytes, dev)
    call("ak_causal_conv1d_bwd", ptr(dx), ptr(dw), ptr(db), ptr(ws), ws_bytes, ptr(x), ptr(w32), ptr(b32), ptr(dy), B, D, T, K, int(bool(silu)), dtype_code(x),
         stream(dev))
    return dx, dw, db


def exported_symbols() -> Sequence[str]:
    return list(SIGNATURES) + ["ak_last_error"]
