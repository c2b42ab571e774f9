"""End-to-end hybrid LM with the B200 kernels swapped in vs the same model with kernels off."""
import pytest
import torch

from conftest import assert_fp32_close

pytestmark = pytest.mark.gpu

TINY = dict(vocab_size=512, d_model=128, n_layers=4, n_heads=4, n_kv_heads=2, ffn_hidden=256, d_state=16)


def _oracle_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
    from oracle import hot_path_oracle as O
    out, _ = O.selective_scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dt=torch.float64)
    return out.to(u.dtype)


def _loss_and_grads(tr, idx, tgt):
    h = tr.model(idx)
    loss = tr.loss_fn(h.reshape(-1, h.shape[-1]), tr.raw.lm_head_weight, tgt.reshape(-1))
    loss.backward()
    return loss.detach(), {k: p.grad.detach().clone() for k, p in tr.raw.named_parameters()}


def test_hybrid_kernels_match_eager_fp32():
    from halo_training.hybrid_lm import HybridConfig
    from halo_training.train_step import HybridTrainer, eager_loss_fn, synthetic_batch
    from kernels.hip.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyLoss
    cfg = HybridConfig(**TINY)
    ce = ChunkedLinearCrossEntropyLoss(chunk_size=128)
    gpu = HybridTrainer(cfg, device=torch.device("cuda"), use_kernels=True, autocast=False,
                        loss_fn=lambda h, w, t: ce(h, w, t))
    cpu = HybridTrainer(cfg, device=torch.device("cpu"), use_kernels=False, autocast=False,
                        scan_fn=_oracle_scan, loss_fn=eager_loss_fn)
    idx, tgt = synthetic_batch(2, 300, cfg.vocab_size, seed=3, device="cpu")
    lg, gg = _loss_and_grads(gpu, idx.cuda(), tgt.cuda())
    lc, gc = _loss_and_grads(cpu, idx, tgt)
    assert abs(lg.item() - lc.item()) < 1e-4
    for k in gc:
        assert_fp32_close(gg[k], gc[k], rtol=1e-3, what=k)


def test_hybrid_124m_bf16_step_all_params_get_grads():
    """Full-size model, one bf16 step: finite loss, every parameter gets a finite nonzero grad
    (the reference's autograd-safety check, scripts/test_autokernel_autograd_safety.py:101-112)."""
    from halo_training.hybrid_lm import HybridConfig, count_params
    from halo_training.train_step import HybridTrainer, synthetic_batch
    cfg = HybridConfig()
    tr = HybridTrainer(cfg, device=torch.device("cuda"), use_kernels=True)
    assert 120e6 < count_params(tr.raw) < 135e6
    import autokernel
    assert autokernel.report(tr.raw)["patterns"]["rmsnorm"]["modules_replaced"] == 2 * cfg.n_layers + 1
    idx, tgt = synthetic_batch(2, 1024, cfg.vocab_size, seed=0, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        h = tr.model(idx)
    loss = tr.loss_fn(h.reshape(-1, h.shape[-1]), tr.raw.lm_head_weight, tgt.reshape(-1))
    assert torch.isfinite(loss) and abs(loss.item() - 10.83) < 0.5  # ~ln(50304) at init
    loss.backward()
    for n, p in tr.raw.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all() and p.grad.abs().sum() > 0, n
    l0 = tr.step(idx, tgt).item()
    for _ in range(3):
        l1 = tr.step(idx, tgt).item()
    assert l1 < l0


def test_residual_chain_matches_unchained_bf16():
    """chain_residuals=True (each residual add inside the next fused add + RMSNorm) against the
    same optimized model without the chain, under bf16 autocast: the hidden stream is the same
    fp32 add rounded once and the gradient accumulation the same fp32 sum, so outputs and
    gradients agree to the last bit (a tight tolerance allows for reordering inside kernels)."""
    import copy

    import autokernel
    from halo_training.hybrid_lm import HybridConfig, HybridLM
    from autokernel._patterns import ResidualPair
    torch.manual_seed(0)
    cfg = HybridConfig(**TINY)
    base = HybridLM(cfg).init_weights(seed=0).cuda()
    for m in base.modules():
        if hasattr(m, "fused_conv"):
            m.fused_conv = True
    plain = autokernel.optimize(copy.deepcopy(base), training=True)
    chained = autokernel.optimize(copy.deepcopy(base), training=True, chain_residuals=True)
    assert autokernel.report(chained)["patterns"]["residual_chain"]["modules_replaced"] == cfg.n_layers - 1
    idx = torch.randint(0, cfg.vocab_size, (2, 256), device="cuda")
    outs = []
    for m in (plain, chained):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            h = m(idx)
            if m is chained:  # intermediate blocks hand on pairs
                with torch.no_grad():
                    assert isinstance(m.layers[0](m.embed(idx)), ResidualPair)
        assert torch.is_tensor(h)
        h.float().square().mean().backward()
        outs.append((h.detach(), {n: p.grad.detach().clone() for n, p in m.named_parameters()}))
    torch.testing.assert_close(outs[1][0], outs[0][0], rtol=0, atol=0)
    for n, g in outs[0][1].items():
        torch.testing.assert_close(outs[1][1][n], g, rtol=1e-5, atol=1e-7, msg=n)


def test_cuda_graph_step_matches_eager():
    """HybridTrainer(cuda_graph=True): eager warm-up calls, then one captured step replayed per
    call; one optimizer step per call, and the loss curve follows the eager trainer's (within
    the run-to-run noise of the atomics-based reductions)."""
    from halo_training.hybrid_lm import HybridConfig
    from halo_training.train_step import HybridTrainer, synthetic_batch
    cfg = HybridConfig(**TINY)
    idx, tgt = synthetic_batch(4, 256, cfg.vocab_size, seed=7, device="cuda")
    curves = []
    for graph in (False, True):
        tr = HybridTrainer(cfg, device=torch.device("cuda"), use_kernels=True, seed=0, cuda_graph=graph)
        curves.append([tr.step(idx, tgt).item() for _ in range(tr.graph_warmup + 4)])
        if graph:
            assert tr._graph is not None
            assert tr.opt.state[next(iter(tr.raw.parameters()))]["step"].item() == tr.graph_warmup + 4
    for a, b in zip(*curves):
        assert abs(a - b) < 2e-3 * max(1.0, abs(a)), (curves[0], curves[1])
    assert curves[1][-1] < curves[1][0]
    with pytest.raises(ValueError, match="captured"):
        tr.step(idx[:, :128], tgt[:, :128])  # a captured step keeps its input shape
