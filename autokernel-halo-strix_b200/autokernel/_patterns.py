"""Pattern definitions: detect a module and build its kernel-backed replacement.

`Pattern(name, priority, op_speedup)` with `matches(name, module, model)` /
`apply(name, module, model)` keeps the reference's contract
(autokernel/_patterns.py:22-33).  The pattern set here is the hot-path one:
  * FusedResidualRMSNormPattern (reference _patterns.py:473-485, replacement
    :364-398, block detection :51-56,102-118), priority 100;
  * RMSNormPattern (reference _patterns.py:508-529), priority 50;
  * FusedSwiGLUPattern (reference :545-609), priority 45, packed `w_gate_up`;
  * SiluGateMulPattern (reference :532-542, replacement :180-215), priority 40.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.nn as nn


@dataclass
class Pattern:
    name: str
    priority: int       # higher = applied first
    op_speedup: float   # informational

    def matches(self, name: str, module: nn.Module, model: nn.Module) -> bool:
        raise NotImplementedError

    def apply(self, name: str, module: nn.Module, model: nn.Module) -> nn.Module:
        raise NotImplementedError


# Class names treated as RMSNorm without further checks.
_RMSNORM_CLASS_NAMES = {"RMSNorm", "LlamaRMSNorm", "MistralRMSNorm", "Qwen2RMSNorm", "T5LayerNorm"}


class _RMSNormReplacement(nn.Module):
    """Replacement for an RMSNorm module.

    Keeps the original `weight` Parameter object (state-dict keys and optimizer
    state stay valid, as in the reference _patterns.py:148-153) and routes every
    floating dtype through the autograd-registered custom op
    `torch.ops.autokernel.rmsnorm_eps` with the module's own eps.  (The
    reference runs its kernel only for fp16 inputs, _patterns.py:166-179, and
    with eps fixed at 1e-6.)
    """

    def __init__(self, original: nn.Module):
        super().__init__()
        self.weight = original.weight
        self.eps = float(getattr(original, "eps", 1e-6) or 1e-6)
        import kernels.hip._torch_ops  # noqa: F401  (registers the ops)
        self._op = torch.ops.autokernel.rmsnorm_eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("autokernel RMSNorm replacement needs CUDA tensors")
        return self._op(x, self.weight, self.eps)


class RMSNormPattern(Pattern):
    def __init__(self):
        super().__init__("rmsnorm", priority=50, op_speedup=3.3)

    def matches(self, name: str, module: nn.Module, model: nn.Module) -> bool:
        if isinstance(module, _RMSNormReplacement):
            return False
        if getattr(module, "_native_norm", False):
            return False
        if isinstance(module, nn.LayerNorm):
            return False
        w = getattr(module, "weight", None)
        if not isinstance(w, torch.Tensor) or w.dim() != 1:
            return False
        if isinstance(module, nn.RMSNorm):
            return True
        cls = type(module).__name__
        return cls in _RMSNORM_CLASS_NAMES or (
            hasattr(module, "eps") and getattr(module, "bias", None) is None and cls.lower().endswith("norm"))

    def apply(self, name: str, module: nn.Module, model: nn.Module) -> nn.Module:
        return _RMSNormReplacement(module)


# (attention, attention_norm, feed_forward, ffn_norm) attribute names of a
# pre-norm residual block; the first four are the reference's aliases
# (_patterns.py:51-56), the last one is the hybrid Mamba/attention layer.
_BLOCK_ALIASES = [
    ("attention", "attention_norm", "feed_forward", "ffn_norm"),
    ("self_attn", "input_layernorm", "mlp", "post_attention_layernorm"),
    ("attn", "pre_norm", "ffn", "ffn_norm"),
    ("conv", "pre_norm", "ffn", "ffn_norm"),
    ("mixer", "pre_norm", "ffn", "ffn_norm"),
]


def _find_block_attrs(module: nn.Module):
    """Alias tuple if `module` is a pre-norm residual block, else None; momentum
    blocks (`log_beta`) and modules flagged `_skip_autokernel` are rejected as in
    the reference (_patterns.py:102-118)."""
    if hasattr(module, "log_beta") or getattr(module, "_skip_autokernel", False):
        return None
    for alias in _BLOCK_ALIASES:
        attn, attn_norm, ffn, ffn_norm = alias
        if all(hasattr(module, a) for a in alias) and isinstance(getattr(getattr(module, ffn_norm), "weight", None),
                                                                 torch.Tensor):
            return alias
    return None


class _FusedResidualRMSNormBlockReplacement(nn.Module):
    """x -> hidden = x + attn(attn_norm(x)); out = hidden + ffn(rmsnorm(hidden)),
    with the residual add and the second norm in one kernel
    (`torch.ops.autokernel.fused_res_rmsnorm_eps`, hidden and normed out of one pass).

    Submodules keep their original attribute names, so state-dict keys and
    optimizer state are unchanged.  Extra forward arguments (e.g. freqs_cis in
    the reference's `forward(x, freqs_cis)`) are passed to the attention
    module.  When the residual stream and the attention output differ in dtype
    (autocast), both are promoted to the wider one, which keeps eager
    semantics; the reference instead casts to fp16 (_patterns.py:386-392).
    """

    def __init__(self, original: nn.Module, alias):
        super().__init__()
        self._alias = tuple(alias)
        for a in alias:
            setattr(self, a, getattr(original, a))
        import kernels.hip._torch_ops  # noqa: F401  (registers the ops)
        self._op = torch.ops.autokernel.fused_res_rmsnorm_eps

    def forward(self, x: torch.Tensor, *args, **kwargs) -> torch.Tensor:
        attn, attn_norm, ffn, ffn_norm = (getattr(self, a) for a in self._alias)
        a = attn(attn_norm(x), *args, **kwargs)
        if not a.is_cuda:
            raise RuntimeError("autokernel fused residual RMSNorm needs CUDA tensors")
        dt = torch.promote_types(a.dtype, x.dtype)
        eps = float(getattr(ffn_norm, "eps", 1e-6) or 1e-6)
        hidden, normed = self._op(a.to(dt), x.to(dt), ffn_norm.weight, eps)
        return hidden + ffn(normed)


class FusedResidualRMSNormPattern(Pattern):
    def __init__(self):
        super().__init__("fused_residual_rmsnorm", priority=100, op_speedup=6.6)

    def matches(self, name: str, module: nn.Module, model: nn.Module) -> bool:
        if isinstance(module, _FusedResidualRMSNormBlockReplacement):
            return False
        return _find_block_attrs(module) is not None

    def apply(self, name: str, module: nn.Module, model: nn.Module) -> nn.Module:
        return _FusedResidualRMSNormBlockReplacement(module, _find_block_attrs(module))


# (gate, down, up) projection names of a SwiGLU MLP (reference _patterns.py:46-49)
_SWIGLU_ALIASES = [
    ("w1", "w2", "w3"),
    ("gate_proj", "down_proj", "up_proj"),
]


def _find_swiglu_attrs(module: nn.Module):
    if getattr(module, "_skip_autokernel", False):
        return None
    for alias in _SWIGLU_ALIASES:
        if all(hasattr(module, a) for a in alias) and isinstance(getattr(module, alias[0]), nn.Linear):
            return alias
    return None


class _SiluGateMulReplacement(nn.Module):
    """down(silu(gate(x)) * up(x)) with the activation product in one kernel
    (`torch.ops.autokernel.silu_gate_mul`, autograd-registered) for every dtype.
    Projections keep their attribute names (state dict unchanged)."""

    def __init__(self, original: nn.Module, alias):
        super().__init__()
        self._alias = tuple(alias)
        for a in alias:
            setattr(self, a, getattr(original, a))
        import kernels.hip._torch_ops  # noqa: F401
        self._op = torch.ops.autokernel.silu_gate_mul

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate_p, down_p, up_p = (getattr(self, a) for a in self._alias)
        gate, up = gate_p(x), up_p(x)
        if not gate.is_cuda:
            raise RuntimeError("autokernel SiLU-gate replacement needs CUDA tensors")
        if up.dtype != gate.dtype:
            dt = torch.promote_types(gate.dtype, up.dtype)
            gate, up = gate.to(dt), up.to(dt)
        return down_p(self._op(gate, up))


class SiluGateMulPattern(Pattern):
    def __init__(self):
        super().__init__("silu_gate_mul", priority=40, op_speedup=1.6)

    def matches(self, name: str, module: nn.Module, model: nn.Module) -> bool:
        return not isinstance(module, _SiluGateMulReplacement) and _find_swiglu_attrs(module) is not None

    def apply(self, name: str, module: nn.Module, model: nn.Module) -> nn.Module:
        return _SiluGateMulReplacement(module, _find_swiglu_attrs(module))


class _FusedSwiGLUReplacement(nn.Module):
    """w_down(silu(gate) * up) with gate, up = w_gate_up(x).chunk(2, -1): the
    packed projection output goes to `torch.ops.autokernel.silu_gate_mul_packed`
    as is (no chunk copies) and its gradient comes back as one packed tensor."""

    def __init__(self, original: nn.Module):
        super().__init__()
        self.w_gate_up = original.w_gate_up
        self.w_down = original.w_down
        import kernels.hip._torch_ops  # noqa: F401
        self._op = torch.ops.autokernel.silu_gate_mul_packed

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gu = self.w_gate_up(x)
        if not gu.is_cuda:
            raise RuntimeError("autokernel fused SwiGLU replacement needs CUDA tensors")
        return self.w_down(self._op(gu.contiguous()))


class FusedSwiGLUPattern(Pattern):
    def __init__(self):
        super().__init__("fused_silu_gate_mul", priority=45, op_speedup=1.6)

    def matches(self, name: str, module: nn.Module, model: nn.Module) -> bool:
        return (not isinstance(module, _FusedSwiGLUReplacement) and isinstance(getattr(module, "w_gate_up", None),
                                                                              nn.Linear)
                and hasattr(module, "w_down") and not getattr(module, "_skip_autokernel", False))

    def apply(self, name: str, module: nn.Module, model: nn.Module) -> nn.Module:
        return _FusedSwiGLUReplacement(module)


ALL_PATTERNS: List[Pattern] = [
    FusedResidualRMSNormPattern(),
    RMSNormPattern(),
    FusedSwiGLUPattern(),
    SiluGateMulPattern(),
]
