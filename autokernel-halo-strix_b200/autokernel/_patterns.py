"""Pattern definitions: detect a module and build its kernel-backed replacement.

`Pattern(name, priority, op_speedup)` with `matches(name, module, model)` /
`apply(name, module, model)` keeps the reference's contract
(autokernel/_patterns.py:22-33).  The pattern set here is the hot-path one:
  * FusedResidualRMSNormPattern (reference _patterns.py:473-485, replacement
    :364-398, block detection :51-56,102-118), priority 100;
  * FusedQKVPattern (reference _patterns.py:488-505, replacement :216-361),
    priority 90: one QKV GEMM, RoPE + head-major transpose in one kernel;
  * RMSNormPattern (reference _patterns.py:508-529), priority 50;
  * FusedSwiGLUPattern (reference :545-609), priority 45, packed `w_gate_up`;
  * SiluGateMulPattern (reference :532-542, replacement :180-215), priority 40.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.nn as nn
import torch.nn.functional as F


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


class ResidualPair:
    """Residual stream value base + delta, not yet added.

    Passed between chained pre-norm blocks (`chain_residual_blocks`): the next
    consumer's RMSNorm adds and normalises in one fused pass
    (`autokernel::fused_res_rmsnorm_mixed`), so the add never runs as its own
    kernel and its backward needs no gradient-accumulation add either.
    base: fp32 residual stream; delta: 16-bit block output (autocast).

    Deliberately not a tuple: a caller loop written for blocks that return
    tuples (`h = block(h); if isinstance(h, tuple): h = h[0]`) would keep only
    `base` and silently drop the block output.  Indexing or unpacking a pair
    raises instead.
    """
    __slots__ = ("base", "delta")

    def __init__(self, base: torch.Tensor, delta: torch.Tensor):
        self.base = base
        self.delta = delta

    def __repr__(self) -> str:
        return f"ResidualPair(base={tuple(self.base.shape)} {self.base.dtype}, delta={tuple(self.delta.shape)} {self.delta.dtype})"

    def materialize(self) -> torch.Tensor:
        return self.base + self.delta


def _pair_fusable(pair: ResidualPair) -> bool:
    return (pair.base.dtype == torch.float32 and pair.delta.dtype in (torch.bfloat16, torch.float16)
            and pair.base.is_cuda and torch.is_autocast_enabled("cuda"))


def _norm_weight_eps(norm: nn.Module):
    w = getattr(norm, "weight", None)
    if not isinstance(w, torch.Tensor):
        return None, None
    return w, float(getattr(norm, "eps", 1e-6) or 1e-6)


def _add_and_norm(pair: ResidualPair, norm: nn.Module):
    """(x, norm(x)) for x = pair.base + pair.delta: one fused kernel when the pair is an fp32
    stream plus a 16-bit delta under autocast and `norm` is an RMSNorm, else the add and the
    module."""
    w, eps = _norm_weight_eps(norm)
    if w is not None and _pair_fusable(pair) and isinstance(norm, (_RMSNormReplacement,)):
        import kernels.hip._torch_ops  # noqa: F401
        return torch.ops.autokernel.fused_res_rmsnorm_mixed(pair.delta, pair.base, w, eps)
    x = pair.materialize()
    return x, norm(x)


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
        self._op_mixed = torch.ops.autokernel.rmsnorm_mixed

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(x, ResidualPair):  # the end of a residual chain: add + norm in one pass
            return _add_and_norm(x, self)[1]
        if not x.is_cuda:
            raise RuntimeError("autokernel RMSNorm replacement needs CUDA tensors")
        if x.dtype == torch.float32 and torch.is_autocast_enabled("cuda"):
            lo = torch.get_autocast_dtype("cuda")
            if lo in (torch.bfloat16, torch.float16):
                # fp32 residual stream under autocast: the output goes straight to a GEMM that
                # would cast it to `lo`; write it in `lo` (same single rounding, no cast kernels)
                return self._op_mixed(x, self.weight, self.eps, lo)
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
        self._op_mixed = torch.ops.autokernel.fused_res_rmsnorm_mixed

    # set by chain_residual_blocks: return ResidualPair(hidden, ffn_out) instead of the sum
    _emit_pair = False

    def forward(self, x, *args, **kwargs):
        attn, attn_norm, ffn, ffn_norm = (getattr(self, a) for a in self._alias)
        if isinstance(x, ResidualPair):  # previous block's output, not yet added
            x, h = _add_and_norm(x, attn_norm)
            a = attn(h, *args, **kwargs)
        else:
            a = attn(attn_norm(x), *args, **kwargs)
        if not a.is_cuda:
            raise RuntimeError("autokernel fused residual RMSNorm needs CUDA tensors")
        eps = float(getattr(ffn_norm, "eps", 1e-6) or 1e-6)
        if (x.dtype == torch.float32 and a.dtype in (torch.bfloat16, torch.float16)
                and torch.is_autocast_enabled("cuda")):
            # fp32 residual stream, 16-bit mixer output: hidden stays fp32, normed comes out in the
            # mixer's dtype for the FFN's autocast GEMM (no promotion or cast kernels)
            hidden, normed = self._op_mixed(a, x, ffn_norm.weight, eps)
        else:
            dt = torch.promote_types(a.dtype, x.dtype)
            hidden, normed = self._op(a.to(dt), x.to(dt), ffn_norm.weight, eps)
        f = ffn(normed)
        if self._emit_pair:
            return ResidualPair(hidden, f)
        return hidden + f


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
        self._op = torch.ops.autokernel.silu_gate_mul_nocast  # no fp16 autocast cast of bf16 activations

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


# (q, k, v, o) projection names (reference _patterns.py:41-44)
_QKV_ALIASES = [
    ("wq", "wk", "wv", "wo"),
    ("q_proj", "k_proj", "v_proj", "o_proj"),
]


def _find_qkv_attrs(module: nn.Module):
    if getattr(module, "_skip_autokernel", False):
        return None
    for alias in _QKV_ALIASES:
        if all(hasattr(module, a) for a in alias) and all(isinstance(getattr(module, a), nn.Linear)
                                                          for a in alias):
            return alias
    return None


def _find_complex_freqs(model: nn.Module):
    """Complex `freqs_cis` buffer of the model, if any (reference _patterns.py:133-138)."""
    if model is None:
        return None
    for bname, buf in model.named_buffers():
        if "freqs_cis" in bname and buf.is_complex():
            return buf
    return None


def _rope_theta(module: nn.Module):
    for a in ("rope_theta", "theta"):
        v = getattr(module, a, None)
        if isinstance(v, (int, float)):
            return float(v)
    return None


class _FusedQKVAttentionReplacement(nn.Module):
    """Causal GQA attention with one QKV GEMM and the RoPE kernel.

    forward(x, freqs_cis=None): qkv = x [Wq; Wk; Wv]^T in one GEMM (the
    concatenation is taken from the original Parameters each call, so state
    dict, optimizer state and gradients stay on them); q and k are rotated
    straight out of the packed qkv rows, and v copied, by one strided RoPE pass
    into a token-major buffer (`qkv_rope_split`: no transpose copies, and the
    backward writes one packed d(qkv) with no slice fills or adds); then
    scaled_dot_product_attention(is_causal=True, enable_gqa) and the output
    projection.  RoPE tables: the complex `freqs_cis` argument or model buffer
    (reference :216-361), else cos / sin of the module's `rope_theta`
    (interleaved pairs, theta^(-2i/D)), cached per length and device.
    """

    def __init__(self, original: nn.Module, alias, freqs_cis=None):
        super().__init__()
        self._alias = tuple(alias)
        for a in alias:
            setattr(self, a, getattr(original, a))
        q_proj = getattr(original, alias[0])
        self.n_heads = int(getattr(original, "n_heads", getattr(original, "num_heads", 1)))
        self.n_kv_heads = int(getattr(original, "n_kv_heads", getattr(original, "num_key_value_heads",
                                                                       self.n_heads)))
        self.head_dim = int(getattr(original, "head_dim", q_proj.out_features // self.n_heads))
        self.theta = _rope_theta(original)
        self._freqs = freqs_cis
        self._tables = {}
        import kernels.hip._torch_ops  # noqa: F401
        from kernels.hip._torch_ops import qkv_rope_split
        self._split = qkv_rope_split  # rotated q, k and v as views of one token-major buffer

    def _cos_sin(self, T: int, device, freqs_cis):
        f = freqs_cis if freqs_cis is not None and torch.is_tensor(freqs_cis) and freqs_cis.is_complex() \
            else self._freqs
        if f is not None:
            f = f[:T].to(device)
            return f.real.float().contiguous(), f.imag.float().contiguous()
        key = (T, str(device))
        if key not in self._tables:
            hd = self.head_dim
            inv = 1.0 / (self.theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
            ang = torch.outer(torch.arange(T, device=device, dtype=torch.float32), inv)
            self._tables[key] = (ang.cos(), ang.sin())
        return self._tables[key]

    def forward(self, x: torch.Tensor, freqs_cis=None, **kwargs) -> torch.Tensor:
        wq, wk, wv, wo = (getattr(self, a) for a in self._alias)
        if not x.is_cuda:
            raise RuntimeError("autokernel fused QKV attention needs CUDA tensors")
        B, T, _ = x.shape
        H, KH, hd = self.n_heads, self.n_kv_heads, self.head_dim
        w = torch.cat([wq.weight, wk.weight, wv.weight], dim=0)
        b = None
        if wq.bias is not None or wk.bias is not None or wv.bias is not None:
            b = torch.cat([p.bias if p.bias is not None else p.weight.new_zeros(p.out_features) for p in (wq, wk, wv)])
        qkv = F.linear(x, w, b)
        cos, sin = self._cos_sin(T, x.device, freqs_cis)
        q, k, v = self._split(qkv, cos, sin, H, KH)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=(H != KH))
        return wo(o.transpose(1, 2).reshape(B, T, H * hd))


class FusedQKVPattern(Pattern):
    def __init__(self):
        super().__init__("fused_qkv", priority=90, op_speedup=1.3)

    def matches(self, name: str, module: nn.Module, model: nn.Module) -> bool:
        if isinstance(module, _FusedQKVAttentionReplacement) or _find_qkv_attrs(module) is None:
            return False
        # RoPE needs tables: a theta on the module or a complex freqs_cis buffer on the model
        return _rope_theta(module) is not None or _find_complex_freqs(model) is not None

    def apply(self, name: str, module: nn.Module, model: nn.Module) -> nn.Module:
        return _FusedQKVAttentionReplacement(module, _find_qkv_attrs(module), _find_complex_freqs(model))


def chain_residual_blocks(model: nn.Module) -> int:
    """Chain the residual stream through consecutive fused pre-norm blocks.

    Opt-in (`autokernel.optimize(..., chain_residuals=True)`): in every
    nn.ModuleList whose members are all fused residual blocks, each block but the
    last returns `ResidualPair(hidden, ffn_out)` and the next block's first
    RMSNorm adds and normalises it in one fused kernel.  This assumes the list is
    run as `h = block(h)` in order (as pre-norm decoders do); code that reads the
    intermediate hidden states must not use it.  The last block of a list returns a
    plain tensor, so whatever follows the list sees what it saw before.
    Returns the number of blocks that emit pairs.
    """
    n = 0
    for mod in model.modules():
        if isinstance(mod, nn.ModuleList) and len(mod) > 1 and all(
                isinstance(b, _FusedResidualRMSNormBlockReplacement) for b in mod):
            for b in list(mod)[:-1]:
                b._emit_pair = True
                n += 1
    return n


ALL_PATTERNS: List[Pattern] = [
    FusedResidualRMSNormPattern(),
    FusedQKVPattern(),
    RMSNormPattern(),
    FusedSwiGLUPattern(),
    SiluGateMulPattern(),
]
