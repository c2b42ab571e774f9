"""autokernel.optimize / report / restore / list_patterns on CPU (no kernel calls)."""
import pytest
import torch
import torch.nn as nn

import autokernel
from autokernel._patterns import (FusedResidualRMSNormPattern, FusedSwiGLUPattern, RMSNormPattern,
                                  SiluGateMulPattern, _FusedResidualRMSNormBlockReplacement, _FusedSwiGLUReplacement,
                                  _RMSNormReplacement, _SiluGateMulReplacement)


class RMSNorm(nn.Module):
    def __init__(self, d, eps=1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


class Block(nn.Module):
    def __init__(self, d=16):
        super().__init__()
        self.attention_norm = RMSNorm(d)
        self.proj = nn.Linear(d, d)
        self.ffn_norm = nn.RMSNorm(d, eps=1e-6)
        self.ln = nn.LayerNorm(d)


def test_list_patterns():
    assert autokernel.list_patterns() == ["fused_residual_rmsnorm", "fused_qkv", "rmsnorm", "fused_silu_gate_mul",
                                          "silu_gate_mul"]


def test_optimize_replaces_rmsnorms_and_keeps_parameters(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    m = nn.Sequential(Block(), Block())
    w0 = m[0].attention_norm.weight
    autokernel.optimize(m, training=True)
    assert isinstance(m[0].attention_norm, _RMSNormReplacement)
    assert isinstance(m[1].ffn_norm, _RMSNormReplacement)
    assert isinstance(m[0].ln, nn.LayerNorm)
    assert m[0].attention_norm.weight is w0  # same Parameter: optimizer/state-dict stay valid
    assert m[0].attention_norm.eps == 1e-5 and m[0].ffn_norm.eps == 1e-6
    assert "0.attention_norm.weight" in m.state_dict()
    rep = autokernel.report(m)
    assert rep["status"] == "optimized" and rep["patterns"]["rmsnorm"]["modules_replaced"] == 4
    assert rep["patterns"]["rmsnorm"]["op_speedup"] == "3.3x"
    autokernel.restore(m)
    assert isinstance(m[0].attention_norm, RMSNorm)
    assert autokernel.report(m) == {"status": "not optimized", "patterns": {}}


def test_include_exclude(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    m = Block()
    autokernel.optimize(m, training=True, exclude=["rmsnorm"])
    assert isinstance(m.attention_norm, RMSNorm)
    m2 = Block()
    autokernel.optimize(m2, training=True, include=["rmsnorm"])
    assert isinstance(m2.attention_norm, _RMSNormReplacement)


def test_inference_mode_casts_dtype(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    m = Block()
    autokernel.optimize(m, dtype=torch.bfloat16)
    assert m.proj.weight.dtype == torch.bfloat16 and not m.training


def test_replacement_refuses_cpu(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    m = Block()
    autokernel.optimize(m, training=True)
    try:
        m.attention_norm(torch.zeros(2, 16))
    except RuntimeError as e:
        assert "CUDA" in str(e)
    else:
        raise AssertionError("expected a loud failure on CPU")


def test_pattern_matching_rules():
    p = RMSNormPattern()
    assert p.matches("n", RMSNorm(4), None)
    assert p.matches("n", nn.RMSNorm(4), None)
    assert not p.matches("n", nn.LayerNorm(4), None)
    assert not p.matches("n", nn.Linear(4, 4), None)


class TransformerBlock(nn.Module):
    """Reference-style block: attention / attention_norm / feed_forward / ffn_norm, forward(x, freqs_cis)."""

    def __init__(self, d=16):
        super().__init__()
        self.attention_norm = RMSNorm(d)
        self.attention = nn.Linear(d, d)
        self.ffn_norm = RMSNorm(d, eps=1e-6)
        self.feed_forward = nn.Linear(d, d)


class MomentumBlock(TransformerBlock):
    def __init__(self, d=16):
        super().__init__(d)
        self.log_beta = nn.Parameter(torch.zeros(1))


def test_fused_residual_block_pattern(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    m = nn.Sequential(TransformerBlock(), MomentumBlock())
    keys = set(m.state_dict())
    autokernel.optimize(m, training=True)
    assert isinstance(m[0], _FusedResidualRMSNormBlockReplacement)
    assert not isinstance(m[1], _FusedResidualRMSNormBlockReplacement)  # momentum blocks are rejected
    # the norms inside the replaced block are replaced by the RMSNorm pattern afterwards
    assert isinstance(m[0].attention_norm, _RMSNormReplacement)
    assert set(m.state_dict()) == keys
    rep = autokernel.report(m)
    assert rep["patterns"]["fused_residual_rmsnorm"] == {"modules_replaced": 1, "op_speedup": "6.6x"}
    autokernel.restore(m)
    assert isinstance(m[0], TransformerBlock) and isinstance(m[0].attention_norm, RMSNorm)
    p = FusedResidualRMSNormPattern()
    assert p.matches("b", TransformerBlock(), None) and not p.matches("b", Block(), None)


class SwiGLU(nn.Module):
    def __init__(self, d=16, h=32):
        super().__init__()
        self.w1, self.w2, self.w3 = nn.Linear(d, h), nn.Linear(h, d), nn.Linear(d, h)


class PackedSwiGLU(nn.Module):
    def __init__(self, d=16, h=32):
        super().__init__()
        self.w_gate_up, self.w_down = nn.Linear(d, 2 * h), nn.Linear(h, d)


def test_swiglu_patterns(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    m = nn.Sequential(SwiGLU(), PackedSwiGLU())
    keys = set(m.state_dict())
    autokernel.optimize(m, training=True)
    assert isinstance(m[0], _SiluGateMulReplacement) and isinstance(m[1], _FusedSwiGLUReplacement)
    assert set(m.state_dict()) == keys
    rep = autokernel.report(m)["patterns"]
    assert rep["silu_gate_mul"]["modules_replaced"] == 1 and rep["fused_silu_gate_mul"]["modules_replaced"] == 1
    assert SiluGateMulPattern().matches("s", SwiGLU(), None) and not SiluGateMulPattern().matches("s", Block(), None)
    assert FusedSwiGLUPattern().matches("s", PackedSwiGLU(), None)


def test_residual_chain_marking(monkeypatch):
    """chain_residuals=True marks every fused block of an all-fused ModuleList but the last to
    hand on ResidualPair(hidden, ffn_out); lists with another module, or a single block, are
    left alone; off by default."""
    from autokernel._patterns import ResidualPair, chain_residual_blocks
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)

    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.ModuleList(TransformerBlock() for _ in range(4))
            self.mixed = nn.ModuleList([TransformerBlock(), nn.Linear(16, 16)])
            self.single = nn.ModuleList([TransformerBlock()])

    m = autokernel.optimize(Net(), training=True)
    assert not any(getattr(b, "_emit_pair", False) for b in m.modules())
    m2 = autokernel.optimize(Net(), training=True, chain_residuals=True)
    flags = [b._emit_pair for b in m2.layers]
    assert flags == [True, True, True, False]
    assert not m2.mixed[0]._emit_pair and not m2.single[0]._emit_pair
    assert autokernel.report(m2)["patterns"]["residual_chain"]["modules_replaced"] == 3
    assert chain_residual_blocks(nn.Sequential(nn.Linear(2, 2))) == 0
    p = ResidualPair(torch.ones(2), torch.full((2,), 2.0))
    assert torch.equal(p.materialize(), torch.full((2,), 3.0))
    # not a tuple: code that unwraps tuple outputs (h = h[0]) fails loudly instead of dropping delta
    assert not isinstance(p, tuple)
    with pytest.raises(TypeError):
        p[0]
    with pytest.raises(TypeError):
        base, delta = p


def test_trainer_cuda_graph_flag_ignored_on_cpu():
    """HybridTrainer(cuda_graph=True) on a CPU device runs the plain eager step."""
    from halo_training.hybrid_lm import HybridConfig
    from halo_training.train_step import HybridTrainer, eager_loss_fn, synthetic_batch
    cfg = HybridConfig(vocab_size=64, d_model=32, n_layers=2, n_heads=2, n_kv_heads=1, ffn_hidden=64, d_state=4)
    from oracle import hot_path_oracle as O

    def scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
        return O.selective_scan(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dt=torch.float64)[0].to(u.dtype)

    tr = HybridTrainer(cfg, device=torch.device("cpu"), use_kernels=False, cuda_graph=True, loss_fn=eager_loss_fn,
                       scan_fn=scan)
    assert tr.cuda_graph is False
    idx, tgt = synthetic_batch(1, 16, cfg.vocab_size, seed=0, device="cpu")
    l0 = tr.step(idx, tgt).item()
    assert tr._graph is None and l0 > 0
