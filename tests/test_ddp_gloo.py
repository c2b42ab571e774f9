"""Data-parallel training step host logic on CPU: 2 gloo ranks vs one process.

The model runs with kernels off (CPU oracle scan, eager loss), so this checks
the DDP wiring of HybridTrainer: after one step both ranks hold identical
parameters equal to a single process that saw both ranks' micro-batches.
Also: a rank that raises is reported on the host, not as a hang.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, REPO

TINY = dict(vocab_size=128, d_model=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_hidden=96, d_state=4)


def oracle_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
    from oracle import hot_path_oracle as O
    out, _ = O.selective_scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dt=torch.float32)
    return out.to(u.dtype)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_path, fail_rank):
    sys.path[:0] = [str(PKG), str(REPO)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        from halo_training.hybrid_lm import HybridConfig
        from halo_training.train_step import HybridTrainer, eager_loss_fn, synthetic_batch
        torch.manual_seed(0)
        tr = HybridTrainer(HybridConfig(**TINY), device=torch.device("cpu"), use_kernels=False, ddp=True,
                           scan_fn=oracle_scan, loss_fn=eager_loss_fn, autocast=False, lr=1e-2)
        tr.opt = torch.optim.SGD(tr.raw.parameters(), lr=0.1)  # Adam's first step is sign(g): too noise-sensitive
        idx, tgt = synthetic_batch(2, 16, TINY["vocab_size"], seed=100 + rank, device="cpu")
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        loss = tr.step(idx, tgt)
        torch.save({"loss": loss, "params": {k: v.detach().clone() for k, v in tr.raw.state_dict().items()}},
                   f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_ddp_two_ranks_match_single_process(tmp_path):
    port = _free_port()
    mp.spawn(_worker, args=(2, port, str(tmp_path / "r"), -1), nprocs=2, join=True)
    r0 = torch.load(tmp_path / "r.0")
    r1 = torch.load(tmp_path / "r.1")
    for k in r0["params"]:
        assert torch.equal(r0["params"][k], r1["params"][k]), k

    sys.path[:0] = [str(PKG), str(REPO)]
    from halo_training.hybrid_lm import HybridConfig
    from halo_training.train_step import HybridTrainer, eager_loss_fn, synthetic_batch
    tr = HybridTrainer(HybridConfig(**TINY), device=torch.device("cpu"), use_kernels=False, ddp=False,
                       scan_fn=oracle_scan, loss_fn=eager_loss_fn, autocast=False, lr=1e-2)
    tr.opt = torch.optim.SGD(tr.raw.parameters(), lr=0.1)
    a = synthetic_batch(2, 16, TINY["vocab_size"], seed=100, device="cpu")
    b = synthetic_batch(2, 16, TINY["vocab_size"], seed=101, device="cpu")
    tr.step(torch.cat([a[0], b[0]]), torch.cat([a[1], b[1]]))
    single = tr.raw.state_dict()
    for k, v in r0["params"].items():
        assert torch.allclose(v, single[k], atol=1e-6, rtol=1e-5), k


def test_ddp_rank_failure_is_reported(tmp_path):
    port = _free_port()
    with pytest.raises(Exception):
        mp.spawn(_worker, args=(2, port, str(tmp_path / "f"), 1), nprocs=2, join=True)
