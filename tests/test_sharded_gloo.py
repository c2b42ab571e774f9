"""Row-sharded ops over 2 and 3 gloo ranks on CPU against the unsharded oracle.

Checks the host logic of kernels/sharded.py: the row split, the order of the collectives of the
fused linear + CE (valid count all-reduced before the gradient is scaled, then loss and dW), and
the batch-summed scan / RMSNorm weight gradients.  The kernels are replaced by CPU functions of
the same contract (float64 autograd of the reference math), so no GPU is needed.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from conftest import PKG, REPO


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_linear_ce(hidden, weight, targets, ignore_index, inv_valid):
    """ak_linear_ce_fwdbwd's contract given the global 1 / n_valid: this shard's part of the
    mean loss, its lse, dH of its rows and its part of dW."""
    h = hidden.double().requires_grad_(True)
    w = weight.double().requires_grad_(True)
    logits = h @ w.t()
    loss = F.cross_entropy(logits, targets, ignore_index=ignore_index, reduction="sum") * inv_valid.double()[0]
    loss.backward()
    return loss.detach().float(), torch.logsumexp(logits.detach(), 1).float(), h.grad.float(), w.grad.float()


def _cpu_rmsnorm_bwd(x, w, dy, eps):
    from oracle import hot_path_oracle as O
    dx, dw = O.rmsnorm_bwd(x, w, dy, eps)
    return dx.float(), dw.float()


def _case(seed, N=96, D=16, V=40, ignore_every=5):
    g = torch.Generator().manual_seed(seed)
    H = torch.randn(N, D, generator=g)
    W = torch.randn(V, D, generator=g) * 0.3
    t = torch.randint(0, V, (N,), generator=g)
    t[::ignore_every] = -100
    x = torch.randn(N, D, generator=g)
    wn = 1 + 0.02 * torch.randn(D, generator=g)
    dy = torch.randn(N, D, generator=g)
    return H, W, t, x, wn, dy


def _worker(rank, world, port, out_path, ignore_every):
    sys.path[:0] = [str(PKG), str(REPO)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        from kernels import sharded
        H, W, t, x, wn, dy = _case(0, ignore_every=ignore_every)
        loss, lse, dH, dW = sharded.linear_ce_sharded(sharded.local_rows(H), W, sharded.local_rows(t),
                                                      fwdbwd=_cpu_linear_ce)
        dx, dwn = sharded.rmsnorm_bwd_sharded(sharded.local_rows(x), wn, sharded.local_rows(dy),
                                              bwd=_cpu_rmsnorm_bwd)
        g = [torch.full((2, 3), float(rank + 1)), torch.ones(2), None, torch.ones(3) * (rank + 1)]
        sg = sharded.selective_scan_bwd_sharded((None, None, g[0], None, None, g[1], None, g[3]))
        torch.save({"loss": loss, "lse": lse, "dH": dH, "dW": dW, "dx": dx, "dwn": dwn,
                    "dA": sg[2], "dD": sg[5], "dbias": sg[7]}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,ignore_every", [(2, 5), (3, 5), (2, 1)])
def test_sharded_ops_match_unsharded(tmp_path, world, ignore_every):
    """world=3 gives ragged shards (96 rows: 32 each, and the split helper's remainder path is
    covered by test_shard_range); ignore_every=1 ignores every row (loss 0, zero gradients)."""
    port = _free_port()
    mp.spawn(_worker, args=(world, port, str(tmp_path / "r"), ignore_every), nprocs=world, join=True)
    sys.path[:0] = [str(PKG), str(REPO)]
    from oracle import hot_path_oracle as O
    H, W, t, x, wn, dy = _case(0, ignore_every=ignore_every)
    parts = [torch.load(f"{tmp_path / 'r'}.{r}") for r in range(world)]
    if ignore_every == 1:
        rl, rdh, rdw = torch.zeros(()), torch.zeros_like(H), torch.zeros_like(W)
    else:
        rl, rdh, rdw = O.linear_ce(H, W, t)
    for p in parts:  # loss and dW are global on every rank
        torch.testing.assert_close(p["loss"].double().reshape(()), rl.double(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(p["dW"].double(), rdw.double(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(p["dA"], sum(torch.full((2, 3), float(r + 1)) for r in range(world)))
        torch.testing.assert_close(p["dD"], torch.ones(2) * world)
    torch.testing.assert_close(torch.cat([p["dH"] for p in parts]).double(), rdh.double(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(torch.cat([p["lse"] for p in parts]).double(),
                               torch.logsumexp(H.double() @ W.double().t(), 1), rtol=1e-5, atol=1e-5)
    rdx, rdwn = O.rmsnorm_bwd(x, wn, dy, 1e-6)
    torch.testing.assert_close(torch.cat([p["dx"] for p in parts]).double(), rdx, rtol=1e-5, atol=1e-5)
    for p in parts:
        torch.testing.assert_close(p["dwn"].double(), rdwn, rtol=1e-5, atol=1e-5)


def test_shard_range():
    sys.path[:0] = [str(PKG), str(REPO)]
    from kernels.sharded import shard_range
    for n in (0, 1, 7, 8, 96, 32768, 196608):
        for world in (1, 2, 3, 4, 8):
            blocks = [shard_range(n, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
            sizes = [e - s for s, e in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)
