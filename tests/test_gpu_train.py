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


def _torch_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
    """selective_scan_ref semantics (selective_scan_interface.py:115-181) as a plain fp32 PyTorch
    loop on the inputs' device, autograd through the loop: the kernels-off scan of the eager model."""
    f = torch.float32
    delta = delta.to(f)
    if delta_bias is not None:
        delta = delta + delta_bias[..., None].to(f)
    if delta_softplus:
        delta = torch.nn.functional.softplus(delta)
    batch, dim, L = u.shape
    N = A.shape[1]
    dA = torch.exp(delta.unsqueeze(-1) * A.to(f).view(1, dim, 1, N))
    dBu = delta.unsqueeze(-1) * B.to(f).permute(0, 2, 1).unsqueeze(1) * u.to(f).unsqueeze(-1)
    Cf = C.to(f)
    x = torch.zeros(batch, dim, N, dtype=f, device=u.device)
    ys = []
    for i in range(L):
        x = dA[:, :, i] * x + dBu[:, :, i]
        ys.append(torch.einsum("bdn,bn->bd", x, Cf[:, :, i]))
    out = torch.stack(ys, dim=2)
    if D is not None:
        out = out + u.to(f) * D.to(f).view(-1, 1)
    if z is not None:
        out = out * torch.nn.functional.silu(z.to(f))
    return out.to(u.dtype)


def _grads(tr, idx, tgt, bf16=True):
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
        h = tr.model(idx)
    loss = tr.loss_fn(h.reshape(-1, h.shape[-1]), tr.raw.lm_head_weight, tgt.reshape(-1))
    loss.backward()
    grads = {n: p.grad.float().clone() for n, p in tr.raw.named_parameters()}
    tr.opt.zero_grad(set_to_none=True)
    return loss.item(), grads


def test_hybrid_124m_bf16_benchmarked_step_tracks_eager():
    """The 124M step exactly as bench.py runs it (bf16 autocast, tcgen05 fused linear + CE, fused
    RMSNorm / residual chain / conv / SwiGLU / RoPE kernels, whole-step CUDA graph) against the
    same model with every kernel off (fp32 PyTorch scan loop, F.rms_norm, SDPA, F.cross_entropy,
    eager steps), same seed and batch.  Reference check: scripts/test_autokernel_autograd_safety.py
    :101-112 (every parameter gets a gradient).
    Step 0: the yardstick is the same kernels-off model in fp32 (autocast off).  Both bf16 runs
    (kernels on, kernels off) round their matmul operands to bf16 in different kernels and
    orders, so their gradients scatter around the fp32 ones by a few percent, parameter by
    parameter, either one ahead (measured: 2e-3 for the kernel path in fp32, about 4e-2 for
    either path in bf16).  Bound: over all parameters together the kernel path's relative L2
    error is at most 1.25 x the eager bf16 one; per parameter at most 3 x it + 1e-2, with cosine
    > 0.99.
    Then 20 AdamW steps on one batch (memorisation, so the loss moves): the losses stay within
    1 % of the eager bf16 curve at every step, and both curves fall."""
    from halo_training.hybrid_lm import HybridConfig
    from halo_training.train_step import HybridTrainer, eager_loss_fn, synthetic_batch
    cfg = HybridConfig()
    dev = torch.device("cuda")
    idx, tgt = synthetic_batch(2, 1024, cfg.vocab_size, seed=100, device="cuda")
    on = HybridTrainer(cfg, device=dev, use_kernels=True, seed=0, cuda_graph=True)
    off = HybridTrainer(cfg, device=dev, use_kernels=False, seed=0, scan_fn=_torch_scan, loss_fn=eager_loss_fn)
    pon, poff = dict(on.raw.named_parameters()), dict(off.raw.named_parameters())
    assert set(pon) == set(poff) and all(torch.equal(pon[k], poff[k]) for k in pon)

    l_on, g_on = _grads(on, idx, tgt)
    l_off, g_off = _grads(off, idx, tgt)
    l_32, g_32 = _grads(off, idx, tgt, bf16=False)
    assert abs(l_on - l_32) < 1e-2 and abs(l_off - l_32) < 1e-2, (l_on, l_off, l_32)
    rows, num_on, num_off, den_all = [], 0.0, 0.0, 0.0
    for name, ref in g_32.items():
        got, eag = g_on[name], g_off[name]
        assert torch.isfinite(got).all() and got.abs().sum() > 0, name
        den = ref.norm().clamp_min(1e-30)
        e_on, e_off = ((got - ref).norm() / den).item(), ((eag - ref).norm() / den).item()
        cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
        rows.append((e_on / max(e_off, 1e-12), name, e_on, e_off, cos))
        num_on += (got - ref).square().sum().item()
        num_off += (eag - ref).square().sum().item()
        den_all += ref.square().sum().item()
        assert e_on <= 3 * e_off + 1e-2 and cos > 0.99, \
            f"{name}: kernels-on error {e_on:.3e}, eager bf16 error {e_off:.3e} (vs fp32), cosine {cos:.5f}"
    tot_on, tot_off = (num_on / den_all) ** 0.5, (num_off / den_all) ** 0.5
    print(f"step-0 gradients vs fp32: all parameters {tot_on:.3e} (kernels on) / {tot_off:.3e} (eager bf16); "
          f"worst ratios {sorted(rows)[-3:]}")
    assert tot_on <= 1.25 * tot_off, (tot_on, tot_off)

    curve_on = [on.step(idx, tgt).item() for _ in range(20)]
    curve_off = [off.step(idx, tgt).item() for _ in range(20)]
    print("loss curves (kernels on, eager bf16):", list(zip(curve_on, curve_off)))
    assert all(abs(a - b) <= 1e-2 * max(1.0, abs(b)) for a, b in zip(curve_on, curve_off)), \
        list(zip(curve_on, curve_off))
    assert curve_on[-1] < curve_on[0] - 0.5 and curve_off[-1] < curve_off[0] - 0.5
