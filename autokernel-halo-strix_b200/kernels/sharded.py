"""Row-sharded execution of the swapped ops over a torch.distributed process group.

One process per GPU.  The rows of every op here are independent, so each rank runs the op on
its own contiguous block of rows and no data moves between ranks, except in the fused
linear + cross-entropy, whose mean reduction and shared weight need one exchange:

* RMSNorm: rows M/k per rank, weight replicated; y and dx stay on their rank.  dW is a sum over
  rows, so `rmsnorm_bwd_sharded` all-reduces its 768 floats when a global dW is wanted.
* Softmax: rows (B*H*L)/k per rank; nothing exchanged.
* Mamba selective scan: batch rows B/k per rank (B, C replicated per batch row, so they shard
  with it); out, du, ddelta, dz, dB, dC stay local; dA, dD and ddelta_bias are sums over the
  batch and are all-reduced by `selective_scan_bwd_sharded` when a global value is wanted.
* Linear + CE (reference chunked_linear_cross_entropy.py:50-175 with the token dimension split
  over ranks, the split the reference's data-parallel trainer makes, scripts/train_ddp.py:228-249):
  the valid-row count is all-reduced first, so every rank scales its rows by the GLOBAL
  1 / n_valid inside the kernel; then the loss (already this shard's part of the global mean) and
  dW (this shard's part of the global sum) are all-reduced.  dH stays local.

Every collective is issued on the current stream right after the kernel that produced its input,
through torch.distributed (NCCL on GPUs, gloo in the CPU tests).  The kernel callables are
parameters so the CPU tests can drive this host logic with a CPU implementation.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def _world(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of rank's block when n rows are split over world ranks: the first n % world
    ranks take one row more, so every row has exactly one owner and blocks are contiguous."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"shard_range: rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_rows(t: torch.Tensor, group=None, dim: int = 0) -> torch.Tensor:
    """This rank's block of t along dim (a view)."""
    world, rank = _world(group)
    s, e = shard_range(t.shape[dim], world, rank)
    return t.narrow(dim, s, e - s)


def _all_reduce(t: torch.Tensor, group) -> torch.Tensor:
    if _world(group)[0] > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def _default_linear_ce(hidden, weight, targets, ignore_index, inv_valid):
    from kernels import _ak
    return _ak.linear_ce_fwdbwd(hidden, weight, targets, ignore_index, inv_valid=inv_valid)


def linear_ce_sharded(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                      ignore_index: int = -100, group=None,
                      fwdbwd: Optional[Callable] = None):
    """Fused linear + mean cross-entropy over this rank's token shard.

    hidden [n_local, D], targets [n_local] are this rank's tokens; weight [V, D] is replicated.
    Returns (loss, lse, dH, dW): loss and dW are the values of the whole (unsharded) batch on
    every rank, lse and dH cover this rank's rows.  Collectives: all-reduce of the valid count
    (one float, before the kernel scales the gradient), of the loss (one float) and of dW.

    fwdbwd(hidden, weight, targets, ignore_index, inv_valid) -> (loss, lse, dH, dW) is the kernel;
    the default is the library's tcgen05 `ak_linear_ce_fwdbwd`."""
    fwdbwd = fwdbwd or _default_linear_ce
    n_valid = (targets != ignore_index).sum(dtype=torch.float32).reshape(1)
    _all_reduce(n_valid, group)
    inv_valid = 1.0 / n_valid.clamp_min(1.0)  # all rows ignored: loss 0 and zero gradients
    loss, lse, dH, dW = fwdbwd(hidden, weight, targets, ignore_index, inv_valid)
    _all_reduce(loss, group)
    if dW is not None:
        _all_reduce(dW, group)
    return loss, lse, dH, dW


def _default_rmsnorm_bwd(x, w, dy, eps):
    from kernels import _ak
    return _ak.rmsnorm_bwd(x, w, dy, eps)


def rmsnorm_bwd_sharded(x: torch.Tensor, w: torch.Tensor, dy: torch.Tensor, eps: float = 1e-6,
                        group=None, global_dw: bool = True, bwd: Optional[Callable] = None):
    """RMSNorm backward of this rank's rows; dW all-reduced to the whole batch's when global_dw."""
    dx, dw = (bwd or _default_rmsnorm_bwd)(x, w, dy, eps)
    if global_dw:
        _all_reduce(dw, group)
    return dx, dw


def selective_scan_bwd_sharded(grads: tuple, group=None) -> tuple:
    """All-reduce the batch-summed gradients (dA, dD, ddelta_bias; None entries skipped) of a
    batch-sharded selective-scan backward.  grads = (du, ddelta, dA, dB, dC, dD, dz, ddelta_bias)
    in the order of selective_scan_fn's inputs; the per-batch-row ones are returned untouched."""
    du, ddelta, dA, dB, dC, dD, dz, dbias = grads
    for t in (dA, dD, dbias):
        if t is not None:
            _all_reduce(t, group)
    return du, ddelta, dA, dB, dC, dD, dz, dbias
