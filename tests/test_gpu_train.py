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
