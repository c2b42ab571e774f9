"""Mamba-style selective scan on B200 with the mamba_ssm 2.3.0 interface.

`selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
delta_softplus=False, return_last_state=False)` and `SelectiveScanFn` keep the
signature and semantics of external/mamba/mamba_ssm/ops/selective_scan_interface.py:23-112
(the reference's GPU path for the hybrid's Mamba blocks, called from
models/amadeus.py:58-79): u, delta, z (batch, dim, L); A (dim, N) fp32;
B, C (batch, N, L) or (batch, G, N, L); D, delta_bias (dim,) fp32; out like u;
last_state (batch, dim, N) fp32, whose gradient is not propagated (as in the
reference).  The forward saves the state every `state_stride()` steps so the
backward recomputes instead of storing the full state tensor.

Supported: real A, input-dependent (3-D/4-D) B and C, N <= 32, dtypes
fp32/bf16/fp16.  Complex A and constant (dim, N) B/C raise NotImplementedError.
"""
import torch

from kernels import _ak


class SelectiveScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                return_last_state=False):
        out, last_state, states = _ak.selective_scan_fwd(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                                                          save_states=True)
        ctx.delta_softplus = bool(delta_softplus)
        ctx.has_D = D is not None
        ctx.has_z = z is not None
        ctx.has_bias = delta_bias is not None
        ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, states)
        ctx.mark_non_differentiable(last_state)
        return out if not return_last_state else (out, last_state)

    @staticmethod
    def backward(ctx, dout, *args):
        u, delta, A, B, C, D, z, delta_bias, states = ctx.saved_tensors
        du, ddelta, dA, dB, dC, dD, dz, dbias = _ak.selective_scan_bwd(
            dout, u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus, states)
        return (du, ddelta, dA.to(A.dtype), dB.to(B.dtype), dC.to(C.dtype),
                dD.to(D.dtype) if ctx.has_D else None,
                dz if ctx.has_z else None,
                dbias.to(delta_bias.dtype) if ctx.has_bias else None,
                None, None)


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                      return_last_state=False):
    """if return_last_state is True, returns (out, last_state); last_state is (batch, dim, dstate)."""
    return SelectiveScanFn.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus, return_last_state)


def state_stride() -> int:
    return _ak.state_stride()
