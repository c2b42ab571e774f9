"""One data-parallel training step of the 124M hybrid with the B200 kernels swapped in.

Mirrors what the reference's `halo_training --optimize-kernels --bf16 --chunked-ce`
(halo_training/trainer.py:117-123, :283-308, :397-438) and its DDP launcher
(scripts/train_ddp.py) do per step: `autokernel.optimize(model, training=True)` (here with
`chain_residuals=True`: each residual add runs inside the next fused add + RMSNorm),
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
                 bucket_cap_mb: int = 64, autocast: Optional[bool] = None, cuda_graph: bool = False):
        self.device = device
        # whole-step CUDA graph (forward, backward, AdamW): the first `graph_warmup` calls run
        # eagerly, the next one captures and replays, every later call replays.  Each call is
        # exactly one optimizer step either way.
        self.cuda_graph = bool(cuda_graph) and device.type == "cuda"
        self.graph_warmup = 11 if ddp else 3  # DDP settles its buckets in its first iterations
        self._graph = None
        self._calls = 0
        model = HybridLM(cfg, scan_fn=scan_fn).init_weights(seed).to(device)
        if use_kernels:
            import autokernel
            model = autokernel.optimize(model, training=True, chain_residuals=True)
            import kernels.hip._torch_ops  # noqa: F401  (torch.ops.autokernel.causal_conv1d_silu)
            for m in model.modules():
                if isinstance(m, MambaBlock):
                    m.fused_conv = True
        self.raw = model
        if ddp:
            from torch.nn.parallel import DistributedDataParallel as DDP
            ids = [device.index] if device.type == "cuda" else None
            if self.cuda_graph:
                # capture-safe DDP: built on the side stream that also runs the eager warm-up
                # steps, as CUDA-graph capture of its all-reduce hooks requires
                s = self._side_stream()
                s.wait_stream(torch.cuda.current_stream(device))
                with torch.cuda.stream(s):
                    model = DDP(model, device_ids=ids, gradient_as_bucket_view=True, bucket_cap_mb=bucket_cap_mb,
                                static_graph=False)
                torch.cuda.current_stream(device).wait_stream(s)
            else:
                model = DDP(model, device_ids=ids, gradient_as_bucket_view=True, bucket_cap_mb=bucket_cap_mb,
                            static_graph=False)
        self.model = model
        fused = device.type == "cuda"
        decay = [p for n, p in self.raw.named_parameters() if p.dim() >= 2]
        no_decay = [p for n, p in self.raw.named_parameters() if p.dim() < 2]
        self.opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                                      {"params": no_decay, "weight_decay": 0.0}],
                                     lr=lr, betas=(0.9, 0.95), eps=1e-8, fused=fused,
                                     capturable=self.cuda_graph)
        self.loss_fn = loss_fn or (kernel_loss_fn() if use_kernels else eager_loss_fn)
        self.autocast = (device.type == "cuda") if autocast is None else autocast

    def _side_stream(self) -> torch.cuda.Stream:
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        return self._side

    def _eager_step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        # the autocast weight-cast cache cannot live across CUDA-graph replays
        with torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.autocast,
                            cache_enabled=not self.cuda_graph):
            h = self.model(idx)
        loss = self.loss_fn(h.reshape(-1, h.shape[-1]), self.raw.lm_head_weight, targets.reshape(-1))
        loss.backward()
        self.opt.step()
        return loss.detach()

    def step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Forward + backward + AdamW on one micro-batch; returns the (device) loss."""
        self._calls += 1
        if not self.cuda_graph or self._calls <= self.graph_warmup:
            if self.cuda_graph:  # warm-up on a side stream, as graph capture requires
                s = self._side_stream()
                s.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(s):
                    loss = self._eager_step(idx, targets)
                    self.opt.zero_grad(set_to_none=True)
                torch.cuda.current_stream(self.device).wait_stream(s)
                return loss
            loss = self._eager_step(idx, targets)
            self.opt.zero_grad(set_to_none=True)
            return loss
        if self._graph is None:
            self._static = (idx.clone(), targets.clone())
            self.opt.zero_grad(set_to_none=True)  # the captured backward allocates and writes the grads
            self._graph = torch.cuda.CUDAGraph()
            # thread-local capture mode: the NCCL watchdog thread may query events meanwhile
            with torch.cuda.graph(self._graph, stream=self._side_stream(), capture_error_mode="thread_local"):
                self._static_loss = self._eager_step(*self._static)
        else:
            if idx.shape != self._static[0].shape or targets.shape != self._static[1].shape:
                raise ValueError(f"HybridTrainer(cuda_graph=True): the step was captured for inputs "
                                 f"{tuple(self._static[0].shape)} / {tuple(self._static[1].shape)}, got "
                                 f"{tuple(idx.shape)} / {tuple(targets.shape)}")
            self._static[0].copy_(idx, non_blocking=True)
            self._static[1].copy_(targets, non_blocking=True)
        self._graph.replay()
        return self._static_loss.clone()


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, device) -> tuple:
    g = torch.Generator().manual_seed(seed)
    tok = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    return tok[:, :-1].contiguous().to(device), tok[:, 1:].contiguous().to(device)
