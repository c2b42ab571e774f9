"""Optimization engine: walk `named_modules()`, match patterns by priority,
replace in place, remember originals for `restore()` and `report()`.

Public functions keep the reference signatures and return shapes
(autokernel/_registry.py:64-178):
  optimize(model, dtype=torch.float16, compile=False, compile_mode="default",
           include=None, exclude=None, training=False) -> model
  report(model) -> {"status", "compiled", "patterns": {name: {"modules_replaced", "op_speedup"}}}
  restore(model) -> model
  list_patterns() -> [names]
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Set

import torch
import torch.nn as nn

from autokernel._patterns import ALL_PATTERNS, Pattern, chain_residual_blocks

_STATE_ATTR = "_autokernel_state"


def _replace_module(model: nn.Module, name: str, new_module: nn.Module) -> None:
    parent = model
    parts = name.split(".")
    for p in parts[:-1]:
        parent = getattr(parent, p)
    setattr(parent, parts[-1], new_module)


def _select_patterns(include: Optional[List[str]], exclude: Optional[List[str]]) -> List[Pattern]:
    pats = list(ALL_PATTERNS)
    if include is not None:
        keep = set(include)
        pats = [p for p in pats if p.name in keep]
    if exclude is not None:
        drop = set(exclude)
        pats = [p for p in pats if p.name not in drop]
    return pats


def optimize(model: nn.Module, dtype: torch.dtype = torch.float16, compile: bool = False,
             compile_mode: str = "default", include: Optional[List[str]] = None,
             exclude: Optional[List[str]] = None, training: bool = False,
             chain_residuals: bool = False) -> nn.Module:
    """Replace every matching module with its kernel-backed version (in place).

    As in the reference: when `training` is False the model is cast to `dtype`
    (complex buffers preserved) and put in eval mode; with `training=True` the
    parameters keep their dtype (mixed precision is left to autocast).  The
    model is moved to the current CUDA device if it is on the CPU.

    chain_residuals (added, off by default): chain the residual stream through
    consecutive fused pre-norm blocks of each nn.ModuleList
    (`chain_residual_blocks`), so each residual add runs inside the next block's
    fused add + RMSNorm kernel.  Only for models that run such a list as
    `h = block(h)` and read no intermediate hidden state.
    """
    if not training:
        saved = {n: b.clone() for n, b in model.named_buffers() if b.is_complex()}
        model = model.to(dtype=dtype)
        dev = next(model.parameters()).device
        for n, b in saved.items():
            parent = model
            parts = n.split(".")
            for p in parts[:-1]:
                parent = getattr(parent, p)
            parent.register_buffer(parts[-1], b.to(dev), persistent=False)
    if torch.cuda.is_available() and any(True for _ in model.parameters()) and not next(model.parameters()).is_cuda:
        model = model.cuda()
    if not training:
        model.eval()

    patterns = _select_patterns(include, exclude)
    patterns.sort(key=lambda p: -p.priority)
    originals: Dict[str, nn.Module] = {}
    applied: Dict[str, int] = {}
    replaced: Set[str] = set()
    for pattern in patterns:
        count = 0
        for name, module in list(model.named_modules()):
            if not name or name in replaced:
                continue
            if pattern.matches(name, module, model):
                try:
                    new = pattern.apply(name, module, model)
                except Exception as e:  # mirror the reference: report and keep going
                    print(f"  autokernel: {pattern.name} failed on {name}: {e}")
                    continue
                originals[name] = module
                _replace_module(model, name, new)
                replaced.add(name)
                count += 1
        if count:
            applied[pattern.name] = count

    if chain_residuals:
        n = chain_residual_blocks(model)
        if n:
            applied["residual_chain"] = n

    if compile:
        try:
            import kernels.hip._torch_ops  # noqa: F401
            model = torch.compile(model) if compile_mode == "default" else torch.compile(model, mode=compile_mode)
        except Exception as e:
            print(f"  autokernel: torch.compile failed: {e}")

    setattr(model, _STATE_ATTR, {"originals": originals, "applied": applied,
                                 "patterns": {p.name: p for p in patterns}, "compiled": compile})
    return model


def report(model: nn.Module) -> Dict[str, Any]:
    state = getattr(model, _STATE_ATTR, None)
    if state is None:
        return {"status": "not optimized", "patterns": {}}
    out = {"status": "optimized", "compiled": state["compiled"], "patterns": {}}
    for name, count in state["applied"].items():
        p = state["patterns"].get(name)
        out["patterns"][name] = {"modules_replaced": count,
                                 "op_speedup": f"{p.op_speedup:.1f}x" if p else "unknown"}
    return out


def restore(model: nn.Module) -> nn.Module:
    state = getattr(model, _STATE_ATTR, None)
    if state is None:
        return model
    for name, original in state["originals"].items():
        _replace_module(model, name, original)
    delattr(model, _STATE_ATTR)
    return model


def list_patterns() -> List[str]:
    return [p.name for p in ALL_PATTERNS]
