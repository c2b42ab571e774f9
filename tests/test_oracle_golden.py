"""The CPU oracle reproduces the reference's own outputs (golden fixtures)."""
import numpy as np
import pytest
import torch

from conftest import assert_fp32_close, golden
from oracle import hot_path_oracle as O

T = torch.from_numpy


def test_rmsnorm_golden():
    g = golden("rmsnorm")
    y = O.rmsnorm_fwd(T(g["x"]), T(g["w"]), float(g["eps"]))
    assert_fp32_close(y, g["y"], 1e-6, "y")
    dx, dw = O.rmsnorm_bwd(T(g["x"]), T(g["w"]), T(g["dy"]), float(g["eps"]))
    assert_fp32_close(dx, g["dx_autograd"], 1e-6, "dx vs autograd of rmsnorm_ref")
    for ref in ("autograd", "fallback"):
        assert_fp32_close(dw, g[f"dw_{ref}"], 1e-6, f"dw vs {ref}")


def test_reference_rmsnorm_fallback_dx_differs_by_missing_rstd():
    """The reference's fp32 backward fallback (kernels/hip/_torch_ops.py:94) computes
    gn*r - normed*mean(gn*normed), dropping a factor r from the second term; the
    autograd of rmsnorm_ref and the reference's HIP kernel
    (kernels/hip/rmsnorm_backward.py:165-166) both use r*(gn - normed*mean(gn*normed)).
    The oracle follows the latter; this test pins the explanation of the gap."""
    g = golden("rmsnorm")
    x, w, dy = (T(g[k]).double() for k in ("x", "w", "dy"))
    r = (x.pow(2).mean(-1, keepdim=True) + float(g["eps"])).rsqrt()
    normed, gn = x * r, dy * w
    fallback = gn * r - normed * (gn * normed).sum(-1, keepdim=True) / x.shape[-1]
    assert_fp32_close(fallback, g["dx_fallback"], 1e-6, "fallback formula")
    assert (torch.from_numpy(g["dx_fallback"]).double() - torch.from_numpy(g["dx_autograd"]).double()).abs().max() > 1e-3


def test_softmax_golden():
    g = golden("softmax")
    y = O.softmax_fwd(T(g["x"]))
    assert_fp32_close(y, g["y"], 1e-6, "y")
    dx = O.softmax_bwd(T(g["y"]), T(g["dy"]))
    assert_fp32_close(dx, g["dx"], 1e-6, "dx")


def test_scan1_golden():
    g = golden("scan1")
    args = [T(g[k]) for k in ("dA", "dBx", "C", "D", "x")]
    y = O.scan1_fwd(*args)
    # the reference forward (amadeus chunked scan) works in fp32 log-space: 1e-5 relative
    assert_fp32_close(y, g["y"], 1e-5, "y")
    grads = O.scan1_bwd(*args, T(g["gy"]))
    for name, got in zip(("gdA", "gdBx", "gC", "gD", "gx"), grads):
        assert_fp32_close(got, g[name], 1e-6, name)


@pytest.mark.parametrize("groups", [1, 2])
def test_selective_scan_golden(groups):
    g = golden(f"sscan_g{groups}")
    ins = {k: T(g[k]) for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")}
    out, last, grads = O.selective_scan_grads(ins["u"], ins["delta"], ins["A"], ins["B"], ins["C"], ins["D"],
                                              ins["z"], ins["delta_bias"], True, T(g["dout"]))
    assert_fp32_close(out, g["out"], 1e-5, "out")
    assert_fp32_close(last, g["last_state"], 1e-5, "last_state")
    for k, v in grads.items():
        assert_fp32_close(v, g["d" + k], 1e-5, "d" + k)


@pytest.mark.parametrize("case,kw", [("plain", {}), ("softcap", dict(softcap=5.0)), ("ls", dict(label_smoothing=0.1)),
                                     ("zloss", dict(z_loss_weight=1e-2)),
                                     ("all", dict(softcap=7.0, label_smoothing=0.05, z_loss_weight=1e-3))])
def test_ce_golden(case, kw):
    g = golden("ce")
    loss, _, grad = O.ce_mean(T(g["logits"]), T(g["targets"]), **kw)
    assert abs(loss.item() - float(g[f"{case}_loss"])) <= 1e-6 * max(1.0, abs(float(g[f"{case}_loss"])))
    assert_fp32_close(grad, g[f"{case}_grad"], 1e-5, "grad")


def test_ce_rows_matches_ce_mean():
    """The per-row fused-grad restatement agrees with the autograd mean formulation."""
    g = golden("ce")
    x, t = T(g["logits"]), T(g["targets"])
    n = (t != -100).sum().item()
    for kw in (dict(), dict(softcap=5.0), dict(label_smoothing=0.1)):
        losses, _, grad = O.ce_rows(x, t, scale=1.0 / n, **kw)
        loss, _, grad_ref = O.ce_mean(x, t, **kw)
        assert abs(losses.sum().item() / n - loss.item()) < 1e-9
        assert_fp32_close(grad, grad_ref, 1e-9, "grad")


def test_linear_ce_golden():
    g = golden("linear_ce")
    loss, dH, dW = O.linear_ce(T(g["H"]), T(g["W"]), T(g["labels"]))
    assert abs(loss.item() - float(g["loss"])) <= 1e-6 * abs(float(g["loss"]))
    assert_fp32_close(dH, g["dH"], 1e-5, "dH")
    assert_fp32_close(dW, g["dW"], 1e-5, "dW")


@pytest.mark.parametrize("tag", ["k4", "k3"])
@pytest.mark.parametrize("silu", [False, True])
def test_causal_conv1d_golden(tag, silu):
    g = golden("conv1d")
    x, w, b, dy = (torch.from_numpy(g[f"{tag}_{k}"]) for k in ("x", "w", "b", "dy"))
    p = f"{tag}_silu_" if silu else f"{tag}_"
    assert_fp32_close(O.causal_conv1d(x, w, b, silu=silu), g[p + "y"], what="y")
    dx, dw, db = O.causal_conv1d_grads(x, w, b, dy, silu=silu)
    assert_fp32_close(dx, g[p + "dx"], what="dx")
    assert_fp32_close(dw, g[p + "dw"], what="dw")
    assert_fp32_close(db, g[p + "db"], what="db")


def test_fused_res_rmsnorm_golden():
    g = golden("fused_res")
    x, r, w, gh, gn = (torch.from_numpy(g[k]) for k in ("x", "residual", "w", "grad_hidden", "grad_normed"))
    h, y = O.fused_res_rmsnorm(x, r, w)
    assert_fp32_close(h, g["hidden"], what="hidden")
    for k in ("normed", "single", "ref_fn"):
        assert_fp32_close(y, g[k], what=k)
    dx, dw = O.fused_res_rmsnorm_bwd(torch.from_numpy(g["hidden"]), w, gh, gn)
    assert_fp32_close(dx, g["dx_autograd"], what="dx")
    assert_fp32_close(dx, g["dres_autograd"], what="dres")
    for k in ("dw_autograd", "dw_op", "dw_kfn"):
        assert_fp32_close(dw, g[k], what=k)


def test_reference_fused_res_fallback_dx_differs_by_missing_rstd():
    """Pins a reference bug: the fp32 branches of _fused_res_rmsnorm_backward
    (kernels/hip/_torch_ops.py:285) and fused_residual_rmsnorm_backward.kernel_fn
    (:277) drop the outer rstd on the mean term, unlike the fp16 HIP kernel
    (:169-170) and autograd.  The oracle follows the HIP kernel and autograd."""
    g = golden("fused_res")
    h = torch.from_numpy(g["hidden"]).double()
    w, gh, gn = (torch.from_numpy(g[k]).double() for k in ("w", "grad_hidden", "grad_normed"))
    r = (h.pow(2).mean(-1, keepdim=True) + 1e-6).rsqrt()
    nh = h * r
    gs = gn * w
    buggy = gh + gs * r - nh * (gs * nh).sum(-1, keepdim=True) / h.shape[-1]
    for k in ("dx_op", "dres_op", "dx_kfn", "dres_kfn"):
        assert_fp32_close(buggy, g[k], rtol=1e-5, what=k)
    assert (torch.from_numpy(g["dx_op"]).double() - torch.from_numpy(g["dx_autograd"]).double()).abs().max() > 1e-3


def test_silu_gate_mul_golden():
    g = golden("silu_gate")
    gate, up, dy = (torch.from_numpy(g[k]) for k in ("gate", "up", "dy"))
    assert_fp32_close(O.silu_gate_mul(gate, up), g["y"], what="y")
    dg, du = O.silu_gate_mul_bwd(gate, up, dy)
    for k in ("dgate_op", "dgate_kfn", "dgate_autograd"):
        assert_fp32_close(dg, g[k], what=k)
    for k in ("dup_op", "dup_kfn", "dup_autograd"):
        assert_fp32_close(du, g[k], what=k)


def test_rope_golden():
    g = golden("rope")
    x, c, s, dy = (torch.from_numpy(g[k]) for k in ("x", "cos", "sin", "dy"))
    assert_fp32_close(O.rope(x, c, s), g["y"], what="y (kernel_fn_fp32)")
    assert_fp32_close(O.rope(x, c, s), g["y_ref"], what="y (rotary_embedding_ref)")
    assert_fp32_close(O.rope_bwd(dy, c, s), g["dx_autograd"], what="dx")


def test_reference_rope_backward_rejects_its_own_tables():
    """Pins a reference bug: _rotary_backward (kernels/hip/_torch_ops.py:140-162) uses the
    rotate-half pairing with full-width tables, so with the forward's (N, D/2) tables it
    raises instead of returning the gradient.  The oracle is the autograd of the forward."""
    assert bool(golden("rope")["ref_bwd_raises"])
