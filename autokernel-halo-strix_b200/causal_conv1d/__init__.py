"""`causal_conv1d_fn` backed by the B200 depthwise causal conv1d kernels.

Drop-in for the `causal_conv1d` package (Dao-AILab causal-conv1d) as the
reference imports it (kernels/hip/_torch_ops.py:878-882, models with
`from causal_conv1d import causal_conv1d_fn`): x (batch, dim, seqlen),
weight (dim, width), bias (dim,) or None, activation None / "silu" / "swish".
seq_idx, initial_states and final-state outputs are not supported and raise.
"""
from typing import Optional

import torch

import kernels.hip._torch_ops  # noqa: F401  (registers torch.ops.autokernel.causal_conv1d*)

__all__ = ["causal_conv1d_fn"]


def causal_conv1d_fn(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                     seq_idx=None, initial_states=None, return_final_states: bool = False,
                     final_states_out=None, activation: Optional[str] = None) -> torch.Tensor:
    if seq_idx is not None or initial_states is not None or return_final_states or final_states_out is not None:
        raise NotImplementedError("causal_conv1d_fn: seq_idx / initial / final states are not supported")
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError(f"causal_conv1d_fn: activation {activation!r}")
    if activation is None:
        return torch.ops.autokernel.causal_conv1d(x, weight, bias)
    return torch.ops.autokernel.causal_conv1d_silu(x, weight, bias)
