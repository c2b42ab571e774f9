"""Pattern definitions: detect a module and build its kernel-backed replacement.

`Pattern(name, priority, op_speedup)` with `matches(name, module, model)` /
`apply(name, module, model)` keeps the reference's contract
(autokernel/_patterns.py:22-33).  The pattern set here is the hot-path one:
RMSNorm (reference RMSNormPattern, _patterns.py:508-529).
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


ALL_PATTERNS: List[Pattern] = [
    RMSNormPattern(),
]
