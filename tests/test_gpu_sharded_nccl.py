"""Row-sharded ops over 2 NCCL ranks (one process per GPU) against the unsharded kernels.

kernels/sharded.py on real GPUs: the fused linear + CE with the global valid count, the loss and
dW all-reduced; the RMSNorm backward with dW all-reduced; the selective-scan backward with dA,
dD and ddelta_bias summed over the batch shards.  Each rank checks its results against the
unsharded call of the same kernels on its own GPU (same seeded inputs).  Skipped with fewer
than two GPUs.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, REPO

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, errfile):
    sys.path[:0] = [str(PKG), str(REPO)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from kernels import _ak, sharded
        g = torch.Generator().manual_seed(5)
        # linear + CE: 4096 tokens, 5 % ignored
        N, D, V = 4096, 256, 8192
        H = torch.randn(N, D, generator=g).to(torch.bfloat16).to(dev)
        W = (torch.randn(V, D, generator=g) * 0.05).to(torch.bfloat16).to(dev)
        lab = torch.randint(0, V, (N,), generator=g)
        lab[torch.randperm(N, generator=g)[: N // 20]] = -100
        lab = lab.to(dev)
        loss, _, dH, dW = _ak.linear_ce_fwdbwd(H, W, lab)
        sl, _, sdH, sdW = sharded.linear_ce_sharded(sharded.local_rows(H), W, sharded.local_rows(lab))
        _ak.check_status(dev)
        torch.testing.assert_close(sl.reshape(()), loss, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(sdH.float(), sharded.local_rows(dH).float(), rtol=0, atol=1e-6)
        torch.testing.assert_close(sdW.float(), dW.float(), rtol=2e-2, atol=2e-5)
        # RMSNorm backward: dx of this rank's rows, dW of the whole batch
        x = torch.randn(2048, 768, generator=g).to(dev)
        w = (1 + 0.02 * torch.randn(768, generator=g)).to(dev)
        dy = torch.randn(2048, 768, generator=g).to(dev)
        dx, dw = _ak.rmsnorm_bwd(x, w, dy, 1e-6)
        sdx, sdw = sharded.rmsnorm_bwd_sharded(sharded.local_rows(x), w, sharded.local_rows(dy), 1e-6)
        torch.testing.assert_close(sdx, sharded.local_rows(dx), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(sdw, dw, rtol=1e-4, atol=1e-4)
        # selective scan backward, batch rows split over the ranks
        b, dim, L, Ns = 4, 64, 512, 16
        bf = torch.bfloat16
        u = torch.randn(b, dim, L, generator=g).to(bf).to(dev)
        delta = (torch.randn(b, dim, L, generator=g) - 4.6).to(bf).to(dev)
        A = (-torch.arange(1, Ns + 1, dtype=torch.float32).repeat(dim, 1)).to(dev)
        Bm = torch.randn(b, Ns, L, generator=g).to(bf).to(dev)
        Cm = torch.randn(b, Ns, L, generator=g).to(bf).to(dev)
        Dv = torch.rand(dim, generator=g).to(dev)
        z = torch.randn(b, dim, L, generator=g).to(bf).to(dev)
        bias = (torch.rand(dim, generator=g) - 4.0).to(dev)
        dout = torch.randn(b, dim, L, generator=g).to(bf).to(dev)

        def grads(uu, dd, BB, CC, zz, oo):
            _o, _l, states = _ak.selective_scan_fwd(uu, dd, A, BB, CC, Dv, zz, bias, True)
            return _ak.selective_scan_bwd(oo, uu, dd, A, BB, CC, Dv, zz, bias, True, states)

        full = grads(u, delta, Bm, Cm, z, dout)
        loc = [sharded.local_rows(t) for t in (u, delta, Bm, Cm, z, dout)]
        part = sharded.selective_scan_bwd_sharded(grads(*loc))
        for i in (2, 5, 7):  # dA, dD, ddelta_bias: summed over the batch
            ref = full[i]
            err = (part[i] - ref).abs().max().item()
            assert err <= 1e-3 * max(ref.abs().max().item(), 1e-30), (i, err)
        for i in (0, 1, 6):  # du, ddelta, dz: this rank's rows, identical
            torch.testing.assert_close(part[i].float(), sharded.local_rows(full[i]).float(), rtol=0, atol=0)
        torch.cuda.synchronize(dev)
    except Exception as e:  # noqa: BLE001 - reported to the parent process
        with open(f"{errfile}.{rank}", "w") as f:
            f.write(repr(e))
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_ops_over_two_nccl_ranks(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path / "err")), nprocs=2, join=True)
