"""autokernel.optimize / report / restore / list_patterns on CPU (no kernel calls)."""
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
