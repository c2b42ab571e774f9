"""Register the B200 kernels as `torch.library` custom ops (namespace `autokernel`).

Mirrors kernels/hip/_torch_ops.py of the reference:
  * `torch.ops.autokernel.rmsnorm(Tensor x, Tensor weight) -> Tensor`
    (reference _torch_ops.py:56-111: fake = empty like x, autograd grads
    (dx, dw), autocast rule cuda/fp16, eps fixed at 1e-6 as in :70);
  * `torch.ops.autokernel.selective_scan(Tensor dA, Tensor dBx, Tensor C,
    Tensor D, Tensor x) -> Tensor` (reference :312-394, grads
    (d dA, d dBx, dC, dD, dx));
  * `torch.ops.autokernel.fused_res_rmsnorm(x, residual, weight) ->
    (hidden, normed)` (reference :238-303);
  * `torch.ops.autokernel.silu_gate_mul(gate, up) -> y` (reference :181-231);
  * `torch.ops.autokernel.rotary_emb_fp32(x, cos, sin) -> y` (reference
    :112-169);
  * `torch.ops.autokernel.causal_conv1d(x, weight, bias) -> y` (reference
    :883-975).
Added here (no reference counterpart):
  * `autokernel::rmsnorm_eps(x, weight, eps)` — same op with the module's eps
    and no autocast cast, used by the module replacement;
  * `autokernel::softmax(x)` — differentiable row softmax;
  * `autokernel::fused_res_rmsnorm_eps(x, residual, weight, eps)` and
    `autokernel::causal_conv1d_silu(x, weight, bias)`,
    `autokernel::silu_gate_mul_packed(gate_up)`;
  * the backward passes as their own custom ops (`*_bwd`), so torch.compile
    sees opaque nodes in both directions instead of tracing into ctypes calls.

Every op body calls libak_b200.so; there is no PyTorch fallback.  The
reference's `AUTOKERNEL_NO_BWD_HIP` / `disable_hip_backward()` switch selects a
PyTorch backward there; here the backward is always the CUDA custom op, so the
switch is accepted for compatibility and has no effect.
"""
import os
from typing import List, Optional, Tuple

import torch

from kernels import _ak

_USE_BWD_HIP = os.environ.get("AUTOKERNEL_NO_BWD_HIP", "0") != "1"


def _use_hip_backward() -> bool:
    """Kept for API compatibility; the CUDA backward is always used."""
    return True


def disable_hip_backward() -> None:
    """Kept for API compatibility (the backward custom ops are compile-safe)."""
    global _USE_BWD_HIP
    _USE_BWD_HIP = False


RMSNORM_EPS = 1e-6

# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::rmsnorm_bwd", mutates_args=())
def rmsnorm_bwd_op(x: torch.Tensor, weight: torch.Tensor, grad: torch.Tensor, eps: float) -> List[torch.Tensor]:
    x2 = x.reshape(-1, x.shape[-1])
    gx, gw = _ak.rmsnorm_bwd(x2, weight, grad.reshape(-1, grad.shape[-1]), eps, dw_dtype=torch.float32)
    return [gx.view(x.shape), gw.to(weight.dtype)]


@rmsnorm_bwd_op.register_fake
def _(x, weight, grad, eps):
    return [x.new_empty(x.shape), weight.new_empty(weight.shape)]


@torch.library.custom_op("autokernel::rmsnorm", mutates_args=())
def rmsnorm_op(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    return _ak.rmsnorm_fwd(x, weight, RMSNORM_EPS)


@rmsnorm_op.register_fake
def _(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    return x.new_empty(x.shape)


def _rmsnorm_setup(ctx, inputs, output):
    x, weight = inputs
    ctx.save_for_backward(x, weight)
    ctx.eps = RMSNORM_EPS


def _rmsnorm_backward(ctx, grad_output):
    x, weight = ctx.saved_tensors
    gx, gw = torch.ops.autokernel.rmsnorm_bwd(x, weight, grad_output.contiguous(), ctx.eps)
    return gx, gw


rmsnorm_op.register_autograd(_rmsnorm_backward, setup_context=_rmsnorm_setup)
try:
    rmsnorm_op.register_autocast("cuda", torch.float16)
except AttributeError:  # older PyTorch
    pass


@torch.library.custom_op("autokernel::rmsnorm_eps", mutates_args=())
def rmsnorm_eps_op(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return _ak.rmsnorm_fwd(x, weight, eps)


@rmsnorm_eps_op.register_fake
def _(x, weight, eps):
    return x.new_empty(x.shape)


def _rmsnorm_eps_setup(ctx, inputs, output):
    x, weight, eps = inputs
    ctx.save_for_backward(x, weight)
    ctx.eps = eps


def _rmsnorm_eps_backward(ctx, grad_output):
    x, weight = ctx.saved_tensors
    gx, gw = torch.ops.autokernel.rmsnorm_bwd(x, weight, grad_output.contiguous(), ctx.eps)
    return gx, gw, None


rmsnorm_eps_op.register_autograd(_rmsnorm_eps_backward, setup_context=_rmsnorm_eps_setup)

# ---------------------------------------------------------------------------
# Softmax (last dim)
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::softmax_bwd", mutates_args=())
def softmax_bwd_op(y: torch.Tensor, grad: torch.Tensor) -> torch.Tensor:
    return _ak.softmax_bwd(y, grad)


@softmax_bwd_op.register_fake
def _(y, grad):
    return y.new_empty(y.shape)


@torch.library.custom_op("autokernel::softmax", mutates_args=())
def softmax_op(x: torch.Tensor) -> torch.Tensor:
    return _ak.softmax_fwd(x)


@softmax_op.register_fake
def _(x):
    return x.new_empty(x.shape)


def _softmax_setup(ctx, inputs, output):
    ctx.save_for_backward(output)


def _softmax_backward(ctx, grad_output):
    (y,) = ctx.saved_tensors
    return torch.ops.autokernel.softmax_bwd(y, grad_output.contiguous())


softmax_op.register_autograd(_softmax_backward, setup_context=_softmax_setup)

# ---------------------------------------------------------------------------
# Collapsed selective scan
# forward: state[t] = dA[t] * state[t-1] + dBx[t]; y[t] = C[t]*state[t] + D*x[t]
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::selective_scan_bwd", mutates_args=())
def selective_scan_bwd_op(dA: torch.Tensor, dBx: torch.Tensor, C: torch.Tensor, D: torch.Tensor, x: torch.Tensor,
                          grad_y: torch.Tensor) -> List[torch.Tensor]:
    return list(_ak.scan1_bwd(dA, dBx, C, D, x, grad_y.float()))


@selective_scan_bwd_op.register_fake
def _(dA, dBx, C, D, x, grad_y):
    return [dA.new_empty(dA.shape), dBx.new_empty(dBx.shape), C.new_empty(C.shape), D.new_empty(D.shape),
            x.new_empty(x.shape)]


# The forward also saves the 64-step chunk-start states, so the backward skips the pass that
# re-derives them (two of its eleven tensor passes).  `autokernel::selective_scan` keeps the
# reference's schema (one output) as a composite over `selective_scan_save`, which returns
# (y, carries) and owns the autograd rule.
@torch.library.custom_op("autokernel::selective_scan_bwd_carries", mutates_args=())
def selective_scan_bwd_carries_op(dA: torch.Tensor, dBx: torch.Tensor, C: torch.Tensor, D: torch.Tensor,
                                  x: torch.Tensor, grad_y: torch.Tensor, carries: torch.Tensor) -> List[torch.Tensor]:
    return list(_ak.scan1_bwd(dA, dBx, C, D, x, grad_y.float(), carries=carries))


@selective_scan_bwd_carries_op.register_fake
def _(dA, dBx, C, D, x, grad_y, carries):
    return [dA.new_empty(dA.shape), dBx.new_empty(dBx.shape), C.new_empty(C.shape), D.new_empty(D.shape),
            x.new_empty(x.shape)]


_SCAN1_CHUNK = 64  # steps per saved chunk-start state (scan1.cu: kW * kSegB)


@torch.library.custom_op("autokernel::selective_scan_save", mutates_args=())
def selective_scan_save_op(dA: torch.Tensor, dBx: torch.Tensor, C: torch.Tensor, D: torch.Tensor,
                           x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    return _ak.scan1_fwd(dA, dBx, C, D, x, save_carries=True)


@selective_scan_save_op.register_fake
def _(dA, dBx, C, D, x):
    B, L, d = dA.shape
    n = max(B * ((L + _SCAN1_CHUNK - 1) // _SCAN1_CHUNK) * d, 1)
    return dA.new_empty(dA.shape), dA.new_empty((n,), dtype=torch.float32)


def _selective_scan_setup(ctx, inputs, output):
    dA, dBx, C, D, x = inputs
    ctx.save_for_backward(dA, dBx, C, D, x, output[1])


def _selective_scan_backward(ctx, grad_y, _grad_carries):
    dA, dBx, C, D, x, carries = ctx.saved_tensors
    gdA, gdBx, gC, gD, gx = torch.ops.autokernel.selective_scan_bwd_carries(dA, dBx, C, D, x, grad_y.contiguous(),
                                                                          carries)
    return (gdA.to(dA.dtype), gdBx.to(dBx.dtype), gC.to(C.dtype), gD.to(D.dtype), gx.to(x.dtype))


selective_scan_save_op.register_autograd(_selective_scan_backward, setup_context=_selective_scan_setup)

_scan_lib = torch.library.Library("autokernel", "FRAGMENT")
_scan_lib.define("selective_scan(Tensor dA, Tensor dBx, Tensor C, Tensor D, Tensor x) -> Tensor")


def _selective_scan_composite(dA, dBx, C, D, x):
    return torch.ops.autokernel.selective_scan_save(dA, dBx, C, D, x)[0]


_scan_lib.impl("selective_scan", _selective_scan_composite, "CompositeImplicitAutograd")


# ---------------------------------------------------------------------------
# Fused residual add + RMSNorm (dual output) — reference _torch_ops.py:238-303:
# `autokernel::fused_res_rmsnorm(x, residual, weight) -> (hidden, normed)`, eps
# 1e-6, grads (grad_x, grad_residual = grad_x, grad_weight), autocast cuda/fp16.
# `fused_res_rmsnorm_eps` (added) carries the norm module's own eps.
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::fused_res_rmsnorm_bwd", mutates_args=())
def fused_res_rmsnorm_bwd_op(hidden: torch.Tensor, weight: torch.Tensor, grad_hidden: Optional[torch.Tensor],
                             grad_normed: torch.Tensor, eps: float) -> List[torch.Tensor]:
    dx, dw = _ak.fused_res_rmsnorm_bwd(hidden, weight, grad_hidden, grad_normed, eps)
    return [dx, dw.to(weight.dtype)]


@fused_res_rmsnorm_bwd_op.register_fake
def _(hidden, weight, grad_hidden, grad_normed, eps):
    return [torch.empty_like(hidden), torch.empty_like(weight)]


def _res_setup(ctx, inputs, output):
    x, residual, weight = inputs[:3]
    ctx.eps = inputs[3] if len(inputs) > 3 else RMSNORM_EPS
    ctx.save_for_backward(output[0], weight)


def _res_backward(ctx, grad_hidden, grad_normed):
    hidden, weight = ctx.saved_tensors
    if grad_normed is None:
        grad_normed = torch.zeros_like(hidden)
    dx, dw = fused_res_rmsnorm_bwd_op(hidden, weight, grad_hidden, grad_normed.contiguous(), ctx.eps)
    return dx, dx, dw


def _res_backward_eps(ctx, grad_hidden, grad_normed):
    return (*_res_backward(ctx, grad_hidden, grad_normed), None)


@torch.library.custom_op("autokernel::fused_res_rmsnorm", mutates_args=())
def fused_res_rmsnorm_op(x: torch.Tensor, residual: torch.Tensor,
                         weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    return _ak.fused_res_rmsnorm_fwd(x, residual, weight, RMSNORM_EPS)


@fused_res_rmsnorm_op.register_fake
def _(x, residual, weight):
    return x.new_empty(x.shape), x.new_empty(x.shape)


fused_res_rmsnorm_op.register_autograd(_res_backward, setup_context=_res_setup)
try:
    fused_res_rmsnorm_op.register_autocast("cuda", torch.float16)
except AttributeError:  # pragma: no cover - older torch
    pass


@torch.library.custom_op("autokernel::fused_res_rmsnorm_eps", mutates_args=())
def fused_res_rmsnorm_eps_op(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                             eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    return _ak.fused_res_rmsnorm_fwd(x, residual, weight, eps)


@fused_res_rmsnorm_eps_op.register_fake
def _(x, residual, weight, eps):
    return x.new_empty(x.shape), x.new_empty(x.shape)


fused_res_rmsnorm_eps_op.register_autograd(_res_backward_eps, setup_context=_res_setup)


# ---------------------------------------------------------------------------
# SiLU gate multiply — reference _torch_ops.py:181-231:
# `autokernel::silu_gate_mul(gate, up) -> silu(gate) * up`, grads (d gate, d up),
# autocast cuda/fp16.  `silu_gate_mul_packed(gate_up)` (added) takes the packed
# (..., 2H) projection output and returns one packed (..., 2H) gradient.
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::silu_gate_mul_bwd", mutates_args=())
def silu_gate_mul_bwd_op(gate: torch.Tensor, up: torch.Tensor, grad: torch.Tensor) -> List[torch.Tensor]:
    return list(_ak.silu_gate_mul_bwd(gate, up, grad))


@silu_gate_mul_bwd_op.register_fake
def _(gate, up, grad):
    return [torch.empty_like(gate), torch.empty_like(up)]


@torch.library.custom_op("autokernel::silu_gate_mul", mutates_args=())
def silu_gate_mul_op(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return _ak.silu_gate_mul_fwd(gate, up)


@silu_gate_mul_op.register_fake
def _(gate, up):
    return gate.new_empty(gate.shape)


def _sgm_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _sgm_backward(ctx, grad):
    gate, up = ctx.saved_tensors
    dg, du = silu_gate_mul_bwd_op(gate, up, grad.contiguous())
    return dg, du


silu_gate_mul_op.register_autograd(_sgm_backward, setup_context=_sgm_setup)
try:
    silu_gate_mul_op.register_autocast("cuda", torch.float16)
except AttributeError:  # pragma: no cover - older torch
    pass


# Same op without the fp16 autocast rule (added): the module replacements call this one,
# so bf16 activations under bf16 autocast stay bf16 (no cast copies in and out).
@torch.library.custom_op("autokernel::silu_gate_mul_nocast", mutates_args=())
def silu_gate_mul_nocast_op(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return _ak.silu_gate_mul_fwd(gate, up)


@silu_gate_mul_nocast_op.register_fake
def _(gate, up):
    return gate.new_empty(gate.shape)


silu_gate_mul_nocast_op.register_autograd(_sgm_backward, setup_context=_sgm_setup)


@torch.library.custom_op("autokernel::silu_gate_mul_packed_bwd", mutates_args=())
def silu_gate_mul_packed_bwd_op(gate_up: torch.Tensor, grad: torch.Tensor) -> torch.Tensor:
    H = gate_up.shape[-1] // 2
    out = torch.empty(gate_up.shape, dtype=gate_up.dtype, device=gate_up.device)
    _ak.silu_gate_mul_bwd(gate_up[..., :H], gate_up[..., H:], grad, packed_out=out)
    return out


@silu_gate_mul_packed_bwd_op.register_fake
def _(gate_up, grad):
    return torch.empty_like(gate_up)


@torch.library.custom_op("autokernel::silu_gate_mul_packed", mutates_args=())
def silu_gate_mul_packed_op(gate_up: torch.Tensor) -> torch.Tensor:
    H = gate_up.shape[-1] // 2
    return _ak.silu_gate_mul_fwd(gate_up[..., :H], gate_up[..., H:])


@silu_gate_mul_packed_op.register_fake
def _(gate_up):
    return gate_up.new_empty((*gate_up.shape[:-1], gate_up.shape[-1] // 2))


def _sgmp_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[0])


def _sgmp_backward(ctx, grad):
    (gate_up,) = ctx.saved_tensors
    return silu_gate_mul_packed_bwd_op(gate_up, grad.contiguous())


silu_gate_mul_packed_op.register_autograd(_sgmp_backward, setup_context=_sgmp_setup)


# ---------------------------------------------------------------------------
# Rotary embedding — reference _torch_ops.py:112-169:
# `autokernel::rotary_emb_fp32(x (B, H, N, D), cos, sin) -> y`, interleaved
# pairs, tables (N, D/2) fp32, autocast rule cuda/fp32.  The backward is the
# exact gradient of that forward (rotation by -theta); the reference's backward
# uses the rotate-half pairing instead.
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::rotary_emb_fp32_bwd", mutates_args=())
def rotary_emb_fp32_bwd_op(grad: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return _ak.rope_bwd(grad, cos, sin)


@rotary_emb_fp32_bwd_op.register_fake
def _(grad, cos, sin):
    return grad.new_empty(grad.shape)


@torch.library.custom_op("autokernel::rotary_emb_fp32", mutates_args=())
def rotary_emb_fp32_op(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return _ak.rope_fwd(x, cos, sin)


@rotary_emb_fp32_op.register_fake
def _(x, cos, sin):
    return x.new_empty(x.shape)


def _rope_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[1], inputs[2])


def _rope_backward(ctx, grad):
    cos, sin = ctx.saved_tensors
    return rotary_emb_fp32_bwd_op(grad, cos, sin), None, None


rotary_emb_fp32_op.register_autograd(_rope_backward, setup_context=_rope_setup)
try:
    rotary_emb_fp32_op.register_autocast("cuda", torch.float32)
except AttributeError:  # pragma: no cover - older torch
    pass


# Same rotation without the fp32 autocast rule (added; the arithmetic is fp32 in the kernel
# either way): the fused-QKV replacement keeps q / k in the activation dtype.
@torch.library.custom_op("autokernel::rotary_emb", mutates_args=())
def rotary_emb_op(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return _ak.rope_fwd(x, cos, sin)


@rotary_emb_op.register_fake
def _(x, cos, sin):
    return x.new_empty(x.shape)


rotary_emb_op.register_autograd(_rope_backward, setup_context=_rope_setup)


# Packed QKV split with RoPE (added).  q, k and v come out as (B, heads, T, hd)
# views of one token-major (B, T, W) buffer: q and k rotated (one launch over
# the H + KH heads), v copied.  The backward writes RoPE^-1(dq), RoPE^-1(dk) and
# dv straight into their columns of one packed d(qkv) (three strided launches),
# where autograd of slice views would zero-fill a full-width gradient per slice
# and add them up.
def _head_view(t: torch.Tensor, off: int, nh: int, hd: int) -> torch.Tensor:
    B, T, _ = t.shape
    return t[..., off:off + nh * hd].view(B, T, nh, hd).transpose(1, 2)


class _QKVRopeSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin, n_heads: int, n_kv_heads: int, head_dim: int):
        B, T, W = qkv.shape
        H, KH, hd = n_heads, n_kv_heads, head_dim
        if W != (H + 2 * KH) * hd:
            raise ValueError(f"qkv_rope_split: width {W} != (H + 2 KH) hd = {(H + 2 * KH) * hd}")
        buf = torch.empty_like(qkv, memory_format=torch.contiguous_format)
        _ak.rope_into(_head_view(buf, 0, H + KH, hd), _head_view(qkv, 0, H + KH, hd), cos, sin, 1)
        _ak.rope_into(_head_view(buf, (H + KH) * hd, KH, hd), _head_view(qkv, (H + KH) * hd, KH, hd), None,
                      None, 0)
        ctx.save_for_backward(cos, sin)
        ctx.dims = (H, KH, hd)
        return (_head_view(buf, 0, H, hd), _head_view(buf, H * hd, KH, hd),
                _head_view(buf, (H + KH) * hd, KH, hd))

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin = ctx.saved_tensors
        H, KH, hd = ctx.dims
        g = next(t for t in (dq, dk, dv) if t is not None)
        B, T = g.shape[0], g.shape[2]
        dqkv = torch.empty((B, T, (H + 2 * KH) * hd), dtype=g.dtype, device=g.device)
        for grad, off, nh, mode in ((dq, 0, H, -1), (dk, H * hd, KH, -1), (dv, (H + KH) * hd, KH, 0)):
            dst = _head_view(dqkv, off, nh, hd)
            if grad is None:
                dst.zero_()
            else:
                _ak.rope_into(dst, grad.to(dqkv.dtype), cos, sin, mode)
        return dqkv, None, None, None, None, None


def qkv_rope_split(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_heads: int, n_kv_heads: int):
    """(B, T, (H + 2 KH) hd) packed projection -> rotated q (B, H, T, hd), rotated k and v
    (B, KH, T, hd), all views of one token-major buffer."""
    hd = qkv.shape[-1] // (n_heads + 2 * n_kv_heads)
    return _QKVRopeSplit.apply(qkv, cos, sin, n_heads, n_kv_heads, hd)


# ---------------------------------------------------------------------------
# Mixed-precision RMSNorm (added): an fp32 residual stream under bf16/fp16
# autocast.  The normalised output is written in the autocast dtype (the value
# the next GEMM's autocast cast would produce, rounded once) and the 16-bit
# gradient is consumed directly, so no cast kernels run in either direction.
#   rmsnorm_mixed(x fp32, weight, eps, out_dtype) -> y (out_dtype)
#   fused_res_rmsnorm_mixed(x 16-bit, residual fp32, weight, eps)
#       -> (hidden fp32, normed 16-bit); grads (dx 16-bit, d residual fp32, dw)
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::rmsnorm_mixed_bwd", mutates_args=())
def rmsnorm_mixed_bwd_op(x: torch.Tensor, weight: torch.Tensor, grad: torch.Tensor,
                         eps: float) -> List[torch.Tensor]:
    dx, _, dw = _ak.rmsnorm_bwd_mixed(x, weight, grad, eps)
    return [dx, dw.to(weight.dtype)]


@rmsnorm_mixed_bwd_op.register_fake
def _(x, weight, grad, eps):
    return [torch.empty_like(x), torch.empty_like(weight)]


@torch.library.custom_op("autokernel::rmsnorm_mixed", mutates_args=())
def rmsnorm_mixed_op(x: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
    return _ak.rmsnorm_fwd_mixed(x, weight, eps, out_dtype)


@rmsnorm_mixed_op.register_fake
def _(x, weight, eps, out_dtype):
    return x.new_empty(x.shape, dtype=out_dtype)


def _rmsnorm_mixed_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[0], inputs[1])
    ctx.eps = inputs[2]


def _rmsnorm_mixed_backward(ctx, grad):
    x, w = ctx.saved_tensors
    dx, dw = rmsnorm_mixed_bwd_op(x, w, grad.contiguous(), ctx.eps)
    return dx, dw, None, None


rmsnorm_mixed_op.register_autograd(_rmsnorm_mixed_backward, setup_context=_rmsnorm_mixed_setup)


@torch.library.custom_op("autokernel::fused_res_rmsnorm_mixed_bwd", mutates_args=())
def fused_res_rmsnorm_mixed_bwd_op(hidden: torch.Tensor, weight: torch.Tensor, grad_hidden: Optional[torch.Tensor],
                                   grad_normed: torch.Tensor, eps: float) -> List[torch.Tensor]:
    dres, dx, dw = _ak.rmsnorm_bwd_mixed(hidden, weight, grad_normed, eps, grad_hidden=grad_hidden, want_lo=True)
    return [dx, dres, dw.to(weight.dtype)]


@fused_res_rmsnorm_mixed_bwd_op.register_fake
def _(hidden, weight, grad_hidden, grad_normed, eps):
    return [torch.empty_like(grad_normed), torch.empty_like(hidden), torch.empty_like(weight)]


@torch.library.custom_op("autokernel::fused_res_rmsnorm_mixed", mutates_args=())
def fused_res_rmsnorm_mixed_op(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                               eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    return _ak.fused_res_rmsnorm_fwd_mixed(x, residual, weight, eps)


@fused_res_rmsnorm_mixed_op.register_fake
def _(x, residual, weight, eps):
    return residual.new_empty(residual.shape), x.new_empty(x.shape)


def _res_mixed_setup(ctx, inputs, output):
    ctx.save_for_backward(output[0], inputs[2])
    ctx.eps = inputs[3]
    ctx.lo_dtype = inputs[0].dtype


def _res_mixed_backward(ctx, grad_hidden, grad_normed):
    hidden, weight = ctx.saved_tensors
    if grad_normed is None:
        grad_normed = torch.zeros(hidden.shape, dtype=ctx.lo_dtype, device=hidden.device)
    dx, dres, dw = fused_res_rmsnorm_mixed_bwd_op(hidden, weight, grad_hidden, grad_normed.contiguous(), ctx.eps)
    return dx, dres, dw, None


fused_res_rmsnorm_mixed_op.register_autograd(_res_mixed_backward, setup_context=_res_mixed_setup)


# ---------------------------------------------------------------------------
# Layout changes of the Mamba block (added): (B, T, D) <-> (B, D, T) through the
# tiled transpose kernel instead of `.transpose(1, 2).contiguous()`.
#   transpose_bt(x (B, R, C)) -> (B, C, R) contiguous; its gradient is a transpose.
#   split_transpose(xz (B, T, Dx + Dz), dx) -> (x (B, Dx, T), z (B, Dz, T)); its
#   gradient is written straight into the two halves of one (B, T, Dx + Dz) tensor.
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::transpose_bt", mutates_args=())
def transpose_bt_op(x: torch.Tensor) -> torch.Tensor:
    return _ak.transpose_bt(x)


@transpose_bt_op.register_fake
def _(x):
    return x.new_empty((x.shape[0], x.shape[2], x.shape[1]))


transpose_bt_op.register_autograd(lambda ctx, g: transpose_bt_op(g.contiguous()),
                                  setup_context=lambda ctx, inputs, output: None)


@torch.library.custom_op("autokernel::split_transpose_bwd", mutates_args=())
def split_transpose_bwd_op(gx: torch.Tensor, gz: torch.Tensor) -> torch.Tensor:
    B, Dx, T = gx.shape
    Dz = gz.shape[1]
    out = torch.empty((B, T, Dx + Dz), dtype=gx.dtype, device=gx.device)
    _ak.transpose_into(out[:, :, :Dx], gx.contiguous())
    _ak.transpose_into(out[:, :, Dx:], gz.contiguous())
    return out


@split_transpose_bwd_op.register_fake
def _(gx, gz):
    return gx.new_empty((gx.shape[0], gx.shape[2], gx.shape[1] + gz.shape[1]))


@torch.library.custom_op("autokernel::split_transpose", mutates_args=())
def split_transpose_op(xz: torch.Tensor, dx: int) -> Tuple[torch.Tensor, torch.Tensor]:
    return _ak.transpose_bt(xz[:, :, :dx]), _ak.transpose_bt(xz[:, :, dx:])


@split_transpose_op.register_fake
def _(xz, dx):
    B, T, Dt = xz.shape
    return xz.new_empty((B, dx, T)), xz.new_empty((B, Dt - dx, T))


def _split_transpose_backward(ctx, gx, gz):
    if gx is None:
        gx = torch.zeros(ctx.shapes[0], dtype=ctx.dtype, device=ctx.device)
    if gz is None:
        gz = torch.zeros(ctx.shapes[1], dtype=ctx.dtype, device=ctx.device)
    return split_transpose_bwd_op(gx, gz), None


def _split_transpose_setup(ctx, inputs, output):
    ctx.shapes = (output[0].shape, output[1].shape)
    ctx.dtype, ctx.device = output[0].dtype, output[0].device


split_transpose_op.register_autograd(_split_transpose_backward, setup_context=_split_transpose_setup)


# ---------------------------------------------------------------------------
# Depthwise causal conv1d — reference _torch_ops.py:883-975
# (`autokernel::causal_conv1d(x (B, D, T), weight (D, K), bias (D,))`, fake =
# empty like x, grads (dx, dweight, dbias), autocast rule cuda/fp16).  The
# reference forward is causal_conv1d_fn or F.pad + F.conv1d(groups=D) and its
# backward replays that under autograd; here both directions are the CUDA
# kernels.  `causal_conv1d_silu` (added) fuses the SiLU of the Mamba block.
# ---------------------------------------------------------------------------


@torch.library.custom_op("autokernel::causal_conv1d_bwd", mutates_args=())
def causal_conv1d_bwd_op(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], grad: torch.Tensor,
                         silu: bool) -> List[torch.Tensor]:
    dx, dw, db = _ak.causal_conv1d_bwd(x, weight, bias, grad, silu)
    out = [dx, dw.to(weight.dtype)]
    if db is not None:
        out.append(db.to(bias.dtype))
    return out


@causal_conv1d_bwd_op.register_fake
def _(x, weight, bias, grad, silu):
    out = [torch.empty_like(x), torch.empty_like(weight)]
    if bias is not None:
        out.append(torch.empty_like(bias))
    return out


def _conv_setup(ctx, inputs, output):
    x, weight, bias = inputs[:3]
    ctx.save_for_backward(x, weight, bias)


def _conv_backward(ctx, grad_out, silu):
    x, weight, bias = ctx.saved_tensors
    g = causal_conv1d_bwd_op(x, weight, bias, grad_out.contiguous(), silu)
    return g[0], g[1], (g[2] if bias is not None else None)


@torch.library.custom_op("autokernel::causal_conv1d", mutates_args=())
def causal_conv1d_op(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    return _ak.causal_conv1d_fwd(x, weight, bias, silu=False)


@causal_conv1d_op.register_fake
def _(x, weight, bias):
    return x.new_empty(x.shape)


causal_conv1d_op.register_autograd(lambda ctx, g: _conv_backward(ctx, g, False), setup_context=_conv_setup)
try:
    causal_conv1d_op.register_autocast("cuda", torch.float16)
except AttributeError:  # pragma: no cover - older torch
    pass


@torch.library.custom_op("autokernel::causal_conv1d_silu", mutates_args=())
def causal_conv1d_silu_op(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    return _ak.causal_conv1d_fwd(x, weight, bias, silu=True)


@causal_conv1d_silu_op.register_fake
def _(x, weight, bias):
    return x.new_empty(x.shape)


causal_conv1d_silu_op.register_autograd(lambda ctx, g: _conv_backward(ctx, g, True), setup_context=_conv_setup)
