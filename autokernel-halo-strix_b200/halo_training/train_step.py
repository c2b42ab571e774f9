"""One data-parallel training step of the 124M hybrid with the B200 kernels swapped in.

Mirrors what the reference's `halo_training --optimize-kernels --bf16 --chunked-ce`
(halo_training/trainer.py:117-123, :283-308, :397-438) and its DDP launcher
(scripts/train_ddp.py) do per step: `autokernel.optimize(model, training=True)`,
bf16 autocast forward, fused linear + cross-entropy on the tied LM head,
backward, AdamW step.  Data parallelism is torch DDP over NCCL (bucketed
all-reduce overlapped with the backward) instead of the reference's manual
per-parameter all-reduce applied one step late (train_ddp.py:1570-1582).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from halo_training.hybrid_lm import HybridConfig, HybridLM, MambaBlock


def kernel_loss_fn():
    """Fused linear + CE on the tied head (the B200 kernel path)."""
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    ce = ChunkedLinearCrossEntropyLoss(chunk_size=4096)

    def loss(h, w, targets):
        return ce(h.to(torch.bfloat16), w.to(torch.bfloat16), targets)
    return loss


def eager_loss_fn(h, w, targets):
    """Plain PyTorch reference head (kernels off)."""
    return F.cross_entropy(F.linear(h, w.to(h.dtype)).float(), targets, ignore_index=-100)


class HybridTrainer:
    def __init__(self, cfg: HybridConfig = HybridConfig(), device: torch.device = torch.device("cuda"),
                 use_kernels: bool = True, ddp: bool = False, lr: float = 3e-4, seed: int = 0,
                 scan_fn: Optional[Callable] = None, loss_fn: Optional[Callable] = None,
                 bucket_cap_mb: int = 64, autocast: Optional[bool] = None):
        self.device = device
        model = HybridLM(cfg, scan_fn=scan_fn).init_weights(seed).to(device)
        if use_kernels:
            import autokernel
            model = autokernel.optimize(model, training=True)
            import kernels.hip._torch_ops  # noqa: F401  (torch.ops.autokernel.causal_conv1d_silu)
            for m in model.modules():
                if isinstance(m, MambaBlock):
                    m.fused_conv = True
        self.raw = model
        if ddp:
            from torch.nn.parallel import DistributedDataParallel as DDP
            ids = [device.index] if device.type == "cuda" else None
            model = DDP(model, device_ids=ids, gradient_as_bucket_view=True, bucket_cap_mb=bucket_cap_mb,
                        static_graph=False)
        self.model = model
        fused = device.type == "cuda"
        decay = [p for n, p in self.raw.named_parameters() if p.dim() >= 2]
        no_decay = [p for n, p in self.raw.named_parameters() if p.dim() < 2]
        self.opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                                      {"params": no_decay, "weight_decay": 0.0}],
                                     lr=lr, betas=(0.9, 0.95), eps=1e-8, fused=fused)
        self.loss_fn = loss_fn or (kernel_loss_fn() if use_kernels else eager_loss_fn)
        self.autocast = (device.type == "cuda") if autocast is None else autocast

    def step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Forward + backward + AdamW on one micro-batch; returns the (device) loss."""
        with torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.autocast):
            h = self.model(idx)
        loss = self.loss_fn(h.reshape(-1, h.shape[-1]), self.raw.lm_head_weight, targets.reshape(-1))
        loss.backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach()


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, device) -> tuple:
    g = torch.Generator().manual_seed(seed)
    tok = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    return tok[:, :-1].contiguous().to(device), tok[:, 1:].contiguous().to(device)
