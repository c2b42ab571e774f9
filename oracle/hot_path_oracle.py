"""CPU oracle for the hot-path kernels — TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU (float64 by default), the
algorithms of the reference implementation for every kernel of the hot path.
It is imported only by `tests/`, by `__graft_entry__.smoke()` and by the
`cpu_baseline` / `--impl reference` legs of `bench.py`, always as the checker
or the timed CPU baseline, never as the product path.  The product path
(`autokernel-halo-strix_b200/`) never imports it.

Parity pinning: `tests/golden/make_golden.py` runs the reference's own code
(reference.py, kernels/hip/_torch_ops.py fallbacks, models/amadeus.py
selective_scan_chunked, mamba_ssm selective_scan_ref, kernels/ce_fused.py
fp32 path) on seeded inputs and stores the results in `tests/golden/*.npz`;
`tests/test_oracle_golden.py` checks every function here against them.

Each function cites the reference lines it restates (paths inside the
joelhenwang/autokernel-halo-strix project).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

DEFAULT = torch.float64


def _c(t: Optional[torch.Tensor], dt=DEFAULT) -> Optional[torch.Tensor]:
    return None if t is None else t.detach().to("cpu", dt)


# ---------------------------------------------------------------------------
# RMSNorm — reference.py:26-29 (forward); backward = autograd of the forward, as in
# kernels/hip/rmsnorm_backward.py:60-189 (grad_w as _torch_ops.py:91)
# ---------------------------------------------------------------------------
def rmsnorm_fwd(x, w, eps: float = 1e-6, dt=DEFAULT):
    x, w = _c(x, dt), _c(w, dt)
    rms = torch.sqrt(torch.mean(x ** 2, dim=-1, keepdim=True) + eps)
    return (x / rms) * w


def rmsnorm_bwd(x, w, dy, eps: float = 1e-6, dt=DEFAULT) -> Tuple[torch.Tensor, torch.Tensor]:
    x, w, g = _c(x, dt), _c(w, dt), _c(dy, dt)
    rms_inv = (x.pow(2).mean(-1, keepdim=True) + eps).rsqrt()
    normed = x * rms_inv
    D = x.shape[-1]
    grad_w = (g * normed).sum(dim=tuple(range(g.ndim - 1)))
    gn = g * w
    # r * (gn - normed * mean(gn * normed)): the autograd of reference.rmsnorm_ref and the
    # reference HIP kernel (kernels/hip/rmsnorm_backward.py:165-166).  The fp32 fallback at
    # kernels/hip/_torch_ops.py:94 omits the outer r on the second term.
    grad_x = rms_inv * (gn - normed * (gn * normed).sum(-1, keepdim=True) / D)
    return grad_x, grad_w


# ---------------------------------------------------------------------------
# Softmax — reference.py:15-17 (F.softmax over the last dim) and its autograd
# ---------------------------------------------------------------------------
def softmax_fwd(x, dt=DEFAULT):
    return torch.softmax(_c(x, dt), dim=-1)


def softmax_bwd(y, dy, dt=DEFAULT):
    y, g = _c(y, dt), _c(dy, dt)
    return y * (g - (g * y).sum(-1, keepdim=True))


# ---------------------------------------------------------------------------
# Collapsed selective scan — recurrence of kernels/hip/selective_scan.py:4-6,
# backward of kernels/hip/_torch_ops.py:353-389
# ---------------------------------------------------------------------------
def scan1_fwd(dA, dBx, C, D, x, dt=DEFAULT):
    dA, dBx, C, D, x = (_c(t, dt) for t in (dA, dBx, C, D, x))
    Bsz, L, d = dA.shape
    h = torch.zeros(Bsz, d, dtype=dt)
    ys = []
    for t in range(L):
        h = dA[:, t] * h + dBx[:, t]
        ys.append(C[:, t] * h + D * x[:, t])
    return torch.stack(ys, dim=1) if L else torch.zeros_like(dA)


def scan1_bwd(dA, dBx, C, D, x, gy, dt=DEFAULT):
    dA, dBx, C, D, x, gy = (_c(t, dt) for t in (dA, dBx, C, D, x, gy))
    Bsz, L, d = dA.shape
    states = torch.zeros(Bsz, L + 1, d, dtype=dt)
    for t in range(L):
        states[:, t + 1] = dA[:, t] * states[:, t] + dBx[:, t]
    gdA = torch.zeros_like(dA)
    gdBx = torch.zeros_like(dBx)
    gC = torch.zeros_like(C)
    gD = torch.zeros(d, dtype=dt)
    g = torch.zeros(Bsz, d, dtype=dt)
    for t in range(L - 1, -1, -1):
        gC[:, t] = gy[:, t] * states[:, t + 1]
        g = g + gy[:, t] * C[:, t]
        gD = gD + (gy[:, t] * x[:, t]).sum(0)
        gdA[:, t] = g * states[:, t]
        gdBx[:, t] = g
        g = g * dA[:, t]
    gx = gy * D
    return gdA, gdBx, gC, gD, gx


# ---------------------------------------------------------------------------
# Mamba-style selective scan — selective_scan_ref,
# external/mamba/mamba_ssm/ops/selective_scan_interface.py:115-181 (real A,
# input-dependent B/C of shape (b, N, L) or (b, G, N, L)); backward = autograd.
# ---------------------------------------------------------------------------
def selective_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False, dt=DEFAULT):
    """Returns (out, last_state) in `dt`; differentiable w.r.t. its (float) inputs."""
    u = u.to(dt)
    delta = delta.to(dt)
    if delta_bias is not None:
        delta = delta + delta_bias[..., None].to(dt)
    if delta_softplus:
        delta = F.softplus(delta)
    batch, dim, L = u.shape
    N = A.shape[1]
    Bf, Cf = B.to(dt), C.to(dt)
    if Bf.dim() == 3:
        Bf = Bf.unsqueeze(1)
    if Cf.dim() == 3:
        Cf = Cf.unsqueeze(1)
    Bf = Bf.repeat_interleave(dim // Bf.shape[1], dim=1)  # (b, dim, N, L)
    Cf = Cf.repeat_interleave(dim // Cf.shape[1], dim=1)
    A = A.to(dt)
    deltaA = torch.exp(delta.unsqueeze(-1) * A.view(1, dim, 1, N))          # (b, dim, L, N)
    deltaB_u = delta.unsqueeze(-1) * Bf.permute(0, 1, 3, 2) * u.unsqueeze(-1)  # (b, dim, L, N)
    x = torch.zeros(batch, dim, N, dtype=dt)
    ys = []
    for i in range(L):
        x = deltaA[:, :, i] * x + deltaB_u[:, :, i]
        ys.append((x * Cf[:, :, :, i]).sum(-1))
    y = torch.stack(ys, dim=2) if L else torch.zeros(batch, dim, 0, dtype=dt)
    out = y if D is None else y + u * D.to(dt).view(-1, 1)
    if z is not None:
        out = out * F.silu(z.to(dt))
    return out, x


def selective_scan_grads(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout, dt=DEFAULT):
    """(out, last_state, grads dict) with grads of sum(out * dout) for each given input."""
    named = {"u": u, "delta": delta, "A": A, "B": B, "C": C, "D": D, "z": z, "delta_bias": delta_bias}
    leaves = {k: (v.detach().to("cpu", dt).requires_grad_(True) if v is not None else None) for k, v in named.items()}
    out, last = selective_scan(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
                               leaves["z"], leaves["delta_bias"], delta_softplus, dt)
    (out * _c(dout, dt)).sum().backward()
    grads = {k: v.grad for k, v in leaves.items() if v is not None}
    return out.detach(), last.detach(), grads


# ---------------------------------------------------------------------------
# Cross entropy on logit rows — kernels/ce_fused.py:122-329 (forward, fused
# grad) and :405-488 (tiny backward), z-loss :626-633 / :672-689
# ---------------------------------------------------------------------------
def ce_rows(logits, targets, softcap=0.0, ignore_index=-100, label_smoothing=0.0, scale=1.0, dt=DEFAULT):
    """Returns (losses[B], lse[B], grad[B,V]) with grad = (p - (1-a)onehot - a/V) * cap' * scale."""
    x0 = _c(logits, dt)
    t = targets.detach().cpu().long()
    B, V = x0.shape
    x = softcap * torch.tanh(x0 / softcap) if softcap > 0 else x0
    lse = torch.logsumexp(x, dim=-1)
    valid = t != ignore_index
    tc = t.clamp(0, V - 1)
    xt = x.gather(1, tc.view(-1, 1)).squeeze(1)
    a = label_smoothing
    loss = lse - (1 - a) * xt - a * x.mean(-1) if a > 0 else lse - xt
    loss = torch.where(valid, loss, torch.zeros_like(loss))
    p = torch.exp(x - lse.unsqueeze(1))
    g = p.clone()
    g[torch.arange(B), tc] -= (1 - a)
    g = g - a / V
    if softcap > 0:
        tt = x / softcap
        g = g * (1 - tt * tt)
    g = g * scale
    g[~valid] = 0
    return loss, lse, g


def ce_mean(logits, targets, softcap=0.0, ignore_index=-100, label_smoothing=0.0, z_loss_weight=0.0,
            dt=DEFAULT):
    """Mean loss over valid rows (+ z-loss) and its gradient (ce_full semantics, ce_fused.py:726-785)."""
    x = _c(logits, dt).requires_grad_(True)
    t = targets.detach().cpu().long()
    xc = softcap * torch.tanh(x / softcap) if softcap > 0 else x
    loss = F.cross_entropy(xc, t, ignore_index=ignore_index, label_smoothing=label_smoothing)
    lse = torch.logsumexp(xc, dim=-1)
    if z_loss_weight > 0:
        valid = (t != ignore_index).to(dt)
        n = valid.sum().clamp(min=1.0)
        loss = loss + z_loss_weight * ((lse * valid) ** 2).sum() / n
    loss.backward()
    return loss.detach(), lse.detach(), x.grad


# ---------------------------------------------------------------------------
# Linear + CE — kernels/hip/chunked_linear_cross_entropy.py:55-175 semantics
# (mean over valid rows of CE(H W^T); dH, dW)
# ---------------------------------------------------------------------------
def linear_ce(H, W, targets, ignore_index=-100, softcap=0.0, label_smoothing=0.0, dt=DEFAULT):
    h = _c(H, dt).requires_grad_(True)
    w = _c(W, dt).requires_grad_(True)
    t = targets.detach().cpu().long()
    logits = h @ w.t()
    if softcap > 0:
        logits = softcap * torch.tanh(logits / softcap)
    loss = F.cross_entropy(logits, t, ignore_index=ignore_index, label_smoothing=label_smoothing)
    loss.backward()
    return loss.detach(), h.grad, w.grad


# ---------------------------------------------------------------------------
# Depthwise causal conv1d — autokernel::causal_conv1d, kernels/hip/_torch_ops.py:883-902
# (F.pad(x, (K-1, 0)) then F.conv1d(groups=D)); backward = autograd of it as in
# :910-965.  silu=True appends the SiLU that causal_conv1d_fn(activation="silu")
# applies.
# ---------------------------------------------------------------------------
def causal_conv1d(x, weight, bias=None, silu: bool = False, dt=DEFAULT):
    return _conv1d(_c(x, dt), _c(weight, dt), _c(bias, dt), silu)


def _conv1d(x, w, b, silu):
    K = w.shape[1]
    T = x.shape[-1]
    xp = F.pad(x, (K - 1, 0))
    y = sum(w[None, :, k, None] * xp[..., k:k + T] for k in range(K))
    if b is not None:
        y = y + b[None, :, None]
    return y * torch.sigmoid(y) if silu else y


def causal_conv1d_grads(x, weight, bias, dy, silu: bool = False, dt=DEFAULT):
    """Returns (dx, dweight, dbias or None)."""
    xr = _c(x, dt).requires_grad_(True)
    wr = _c(weight, dt).requires_grad_(True)
    br = _c(bias, dt).requires_grad_(True) if bias is not None else None
    with torch.enable_grad():
        y = _conv1d(xr, wr, br, silu)
        y.backward(_c(dy, dt))
    return xr.grad, wr.grad, (br.grad if br is not None else None)


# ---------------------------------------------------------------------------
# Fused residual add + RMSNorm — reference.fused_residual_add_rmsnorm_ref
# (reference.py:72-78), dual form kernels/hip/fused_residual_add_rmsnorm.py:377-391;
# backward kernels/hip/_torch_ops.py:262-290 (= fused_residual_rmsnorm_backward.py:265-281).
# `round_to`: dtype the sum x + residual is rounded to before the norm (the
# activation dtype; None keeps it exact).
# ---------------------------------------------------------------------------
def fused_res_rmsnorm(x, residual, w, eps: float = 1e-6, round_to=None, dt=DEFAULT):
    if round_to is not None:
        # the activation-dtype add: exact fp32 sum of the two inputs, one rounding
        h = _c((_c(x, torch.float32) + _c(residual, torch.float32)).to(round_to), dt)
    else:
        h = _c(x, dt) + _c(residual, dt)
    return h, rmsnorm_fwd(h, w, eps, dt=dt)


def fused_res_rmsnorm_bwd(hidden, w, grad_hidden, grad_normed, eps: float = 1e-6, dt=DEFAULT):
    """Returns (dx = d residual, dw)."""
    dx, dw = rmsnorm_bwd(hidden, w, grad_normed, eps, dt=dt)
    if grad_hidden is not None:
        dx = dx + _c(grad_hidden, dt)
    return dx, dw


# ---------------------------------------------------------------------------
# SiLU gate multiply — kernels/hip/silu_gate_mul.py:102-118 (fp32 branch
# F.silu(gate) * up); backward kernels/hip/_torch_ops.py:199-218 and
# kernels/hip/silu_gate_mul_backward.py:160-168.
# ---------------------------------------------------------------------------
def silu_gate_mul(gate, up, dt=DEFAULT):
    g, u = _c(gate, dt), _c(up, dt)
    return g * torch.sigmoid(g) * u


def silu_gate_mul_bwd(gate, up, dy, dt=DEFAULT):
    """Returns (d gate, d up)."""
    g, u, gy = _c(gate, dt), _c(up, dt), _c(dy, dt)
    s = torch.sigmoid(g)
    return gy * u * s * (1 + g * (1 - s)), gy * g * s


# ---------------------------------------------------------------------------
# Rotary embedding, interleaved pairs — reference.rotary_embedding_ref
# (reference.py:63-69) = kernels/hip/rotary_embedding.py:258-261,288-291;
# backward = autograd of that forward (rotation by -theta).
# ---------------------------------------------------------------------------
def rope(x, cos, sin, dt=DEFAULT):
    x, c, s = _c(x, dt), _c(cos, dt), _c(sin, dt)
    x1, x2 = x[..., ::2], x[..., 1::2]
    return torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).flatten(-2)


def rope_bwd(dy, cos, sin, dt=DEFAULT):
    g, c, s = _c(dy, dt), _c(cos, dt), _c(sin, dt)
    g1, g2 = g[..., ::2], g[..., 1::2]
    return torch.stack([g1 * c + g2 * s, -g1 * s + g2 * c], dim=-1).flatten(-2)
