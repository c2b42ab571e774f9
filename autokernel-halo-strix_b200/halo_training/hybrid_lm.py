"""124M hybrid LM used for the end-to-end training measurement.

Composed from the reference's pieces (no model of exactly this shape exists
there): RMSNorm / SwiGLU / RoPE as in models/_components.py:25-107, GQA
attention as in models/components/attention.py:69-172, and a mamba_simple-style
Mamba block (external/mamba/mamba_ssm/modules/mamba_simple.py: d_state 16,
d_conv 4, expand 2, dt-bias init :91-99, A = -exp(A_log) :103-110).

Layout: 12 layers at d_model 768 alternating Mamba (even) and GQA attention
(odd; 12 query / 4 KV heads of 64, RoPE), each followed by a SwiGLU MLP of
width 2048, RMSNorm pre-norm everywhere, tied 50304-token embedding.  About
127M parameters.

The kernels enter through the reference's own mechanisms: `autokernel.optimize`
swaps every `RMSNorm`, the Mamba block calls `selective_scan_fn` (injectable
as `scan_fn` so a test can run the same model with a CPU oracle), and the
training step computes the loss with the fused linear + cross-entropy.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class HybridConfig:
    vocab_size: int = 50304
    d_model: int = 768
    n_layers: int = 12
    n_heads: int = 12
    n_kv_heads: int = 4
    ffn_hidden: int = 2048
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    init_std: float = 0.02


class RMSNorm(nn.Module):
    """Plain RMSNorm (models/_components.py:25-39); swapped by autokernel.optimize."""

    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


class SwiGLU(nn.Module):
    def __init__(self, d: int, hidden: int):
        super().__init__()
        self.w1 = nn.Linear(d, hidden, bias=False)
        self.w3 = nn.Linear(d, hidden, bias=False)
        self.w2 = nn.Linear(hidden, d, bias=False)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


def rope_tables(seq: int, head_dim: int, theta: float, device) -> tuple:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    t = torch.arange(seq, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return f.cos(), f.sin()


def apply_rope(x, cos, sin):
    # x: (B, H, T, hd); rotate interleaved pairs (as reference.rotary_embedding_ref)
    x1, x2 = x[..., ::2], x[..., 1::2]
    c, s = cos[None, None].to(x.dtype), sin[None, None].to(x.dtype)
    return torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).flatten(-2)


class GQAAttention(nn.Module):
    def __init__(self, cfg: HybridConfig):
        super().__init__()
        self.n_heads, self.n_kv_heads = cfg.n_heads, cfg.n_kv_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.wq = nn.Linear(cfg.d_model, self.n_heads * self.head_dim, bias=False)
        self.wk = nn.Linear(cfg.d_model, self.n_kv_heads * self.head_dim, bias=False)
        self.wv = nn.Linear(cfg.d_model, self.n_kv_heads * self.head_dim, bias=False)
        self.wo = nn.Linear(self.n_heads * self.head_dim, cfg.d_model, bias=False)
        self.rope_theta = cfg.rope_theta

    def forward(self, x):
        B, T, _ = x.shape
        H, KH, hd = self.n_heads, self.n_kv_heads, self.head_dim
        q = self.wq(x).view(B, T, H, hd).transpose(1, 2)
        k = self.wk(x).view(B, T, KH, hd).transpose(1, 2)
        v = self.wv(x).view(B, T, KH, hd).transpose(1, 2)
        cos, sin = rope_tables(T, hd, self.rope_theta, x.device)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        return self.wo(o.transpose(1, 2).reshape(B, T, H * hd))


class _ChannelMajorLinear(torch.autograd.Function):
    """y[b] = W x[b] for channel-major activations x (B, in, T) -> y (B, out, T).

    The Mamba block's x_proj and dt_proj read and produce the (B, D, T) layout of the conv and
    the scan directly, so neither side needs a transpose copy.  The GEMMs run in the activation
    dtype; the weight gradient sums the batch's per-row products in fp32 (bmm with fp32 output)
    and is returned in the weight's own dtype."""

    @staticmethod
    def forward(ctx, x, weight):
        wc = weight.to(x.dtype)
        ctx.save_for_backward(x, wc)
        ctx.w_dtype = weight.dtype
        return torch.matmul(wc, x)

    @staticmethod
    def backward(ctx, g):
        x, wc = ctx.saved_tensors
        g = g.to(x.dtype)
        dx = torch.matmul(wc.t(), g) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = torch.bmm(g, x.mT, out_dtype=torch.float32).sum(0).to(ctx.w_dtype)
        return dx, dw


def _default_scan():
    from kernels.mamba_scan import selective_scan_fn
    return selective_scan_fn


class MambaBlock(nn.Module):
    """mamba_simple-style mixer: in_proj -> causal depthwise conv -> SiLU -> x_proj
    (dt, B, C) -> dt_proj -> selective scan with SiLU(z) gate -> out_proj."""

    def __init__(self, cfg: HybridConfig, scan_fn: Optional[Callable] = None):
        super().__init__()
        d = cfg.d_model
        self.d_inner = cfg.expand * d
        self.d_state = cfg.d_state
        self.dt_rank = math.ceil(d / 16)
        self.in_proj = nn.Linear(d, 2 * self.d_inner, bias=False)
        self.conv1d = nn.Conv1d(self.d_inner, self.d_inner, cfg.d_conv, groups=self.d_inner,
                                padding=cfg.d_conv - 1, bias=True)
        self.x_proj = nn.Linear(self.d_inner, self.dt_rank + 2 * self.d_state, bias=False)
        self.dt_proj = nn.Linear(self.dt_rank, self.d_inner, bias=True)
        A = torch.arange(1, self.d_state + 1, dtype=torch.float32).repeat(self.d_inner, 1)
        self.A_log = nn.Parameter(torch.log(A))
        self.D = nn.Parameter(torch.ones(self.d_inner))
        self.out_proj = nn.Linear(self.d_inner, d, bias=False)
        self._scan = scan_fn
        # kernel path (set by the trainer with use_kernels): fused causal conv + SiLU and the
        # layout changes through the transpose kernel
        self.fused_conv = False

    def reset_dt(self, generator: Optional[torch.Generator] = None):
        dt_min, dt_max, floor = 1e-3, 1e-1, 1e-4
        std = self.dt_rank ** -0.5
        with torch.no_grad():
            self.dt_proj.weight.uniform_(-std, std, generator=generator)
            dt = torch.exp(torch.rand(self.d_inner, generator=generator) * (math.log(dt_max) - math.log(dt_min))
                           + math.log(dt_min)).clamp(min=floor)
            self.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))

    def forward(self, h):
        if self.fused_conv:
            return self._forward_kernels(h)
        B, T, _ = h.shape
        xz = self.in_proj(h).transpose(1, 2)                    # (B, 2*d_inner, T)
        x, z = xz.chunk(2, dim=1)
        x = F.silu(self.conv1d(x)[..., :T])
        x_dbl = self.x_proj(x.transpose(1, 2))                  # (B, T, dt_rank + 2N)
        dt, Bm, Cm = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        dt = (dt @ self.dt_proj.weight.t().to(dt.dtype)).transpose(1, 2)   # (B, d_inner, T), bias in the scan
        A = -torch.exp(self.A_log.float())
        scan = self._scan or _default_scan()
        y = scan(x.contiguous(), dt.contiguous(), A, Bm.transpose(1, 2).contiguous(),
                 Cm.transpose(1, 2).contiguous(), self.D.float(), z=z.contiguous(),
                 delta_bias=self.dt_proj.bias.float(), delta_softplus=True)
        return self.out_proj(y.transpose(1, 2))

    def _forward_kernels(self, h):
        """Same computation on the kernel path: in_proj's output split and transposed by one
        kernel (torch.ops.autokernel.split_transpose), the fused conv + SiLU, x_proj and dt_proj
        computed channel-major (no transposes), and one transpose of the scan output for
        out_proj."""
        ops = torch.ops.autokernel
        di = self.d_inner
        xz = self.in_proj(h)                                      # (B, T, 2*d_inner)
        x, z = ops.split_transpose(xz, di)                        # (B, d_inner, T) each
        x = ops.causal_conv1d_silu(x, self.conv1d.weight.squeeze(1), self.conv1d.bias)
        x_dbl = _ChannelMajorLinear.apply(x, self.x_proj.weight)  # (B, dt_rank + 2N, T)
        dt, Bm, Cm = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=1)
        dt = _ChannelMajorLinear.apply(dt, self.dt_proj.weight)   # (B, d_inner, T)
        A = -torch.exp(self.A_log.float())
        scan = self._scan or _default_scan()
        y = scan(x, dt, A, Bm, Cm, self.D.float(), z=z,
                 delta_bias=self.dt_proj.bias.float(), delta_softplus=True)
        return self.out_proj(ops.transpose_bt(y))


class HybridLayer(nn.Module):
    def __init__(self, cfg: HybridConfig, mamba: bool, scan_fn=None):
        super().__init__()
        self.pre_norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.mixer = MambaBlock(cfg, scan_fn) if mamba else GQAAttention(cfg)
        self.ffn_norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.ffn = SwiGLU(cfg.d_model, cfg.ffn_hidden)

    def forward(self, h):
        h = h + self.mixer(self.pre_norm(h))
        return h + self.ffn(self.ffn_norm(h))


class HybridLM(nn.Module):
    def __init__(self, cfg: HybridConfig = HybridConfig(), scan_fn: Optional[Callable] = None):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList(HybridLayer(cfg, mamba=(i % 2 == 0), scan_fn=scan_fn)
                                    for i in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps)

    @property
    def lm_head_weight(self):
        return self.embed.weight  # tied

    def init_weights(self, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("A_log") or name.endswith(".D") or "norm" in name or ".conv1d." in name:
                    continue
                if name.endswith("dt_proj.weight") or name.endswith("dt_proj.bias"):
                    continue
                p.normal_(0.0, self.cfg.init_std, generator=g)
            for m in self.modules():
                if isinstance(m, MambaBlock):
                    m.reset_dt(g)
                    bound = m.conv1d.weight.shape[-1] ** -0.5  # PyTorch's default conv init range
                    m.conv1d.weight.uniform_(-bound, bound, generator=g)
                    m.conv1d.bias.uniform_(-bound, bound, generator=g)
        return self

    def forward(self, idx):
        """Returns final hidden states (B, T, d); the loss head is applied by the caller."""
        h = self.embed(idx)
        for layer in self.layers:
            h = layer(h)
        return self.norm(h)


def count_params(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())
