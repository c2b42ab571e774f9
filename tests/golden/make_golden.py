"""Generate the golden fixtures in this directory by running the REFERENCE's own
CPU code paths on seeded inputs.

    python tests/golden/make_golden.py [--reference PATH]

Needs a checkout of joelhenwang/autokernel-halo-strix (default: $AK_REFERENCE, else a
`reference` directory beside this repository; read-only is fine).  Every output stored here comes from the reference's code:
  rmsnorm.npz      reference.rmsnorm_ref (reference.py:26-29) + autograd, and the
                   fp32 branch of kernels/hip/_torch_ops._rmsnorm_backward (:73-97)
  softmax.npz      reference.softmax_ref (reference.py:15-17) + autograd
  scan1.npz        models/amadeus.selective_scan_chunked (forward, :172-264) and
                   kernels/hip/_torch_ops._selective_scan_backward (:335-389)
  sscan_g{1,2}.npz mamba_ssm selective_scan_ref (selective_scan_interface.py:115-181)
                   + autograd (the mamba test's reference, tests/ops/test_selective_scan.py)
  ce.npz           kernels/ce_fused.ce_full fp32 path (:755-777) + autograd, cases
                   plain / softcap / label smoothing / ignore / z-loss
  conv1d.npz       kernels/hip/_torch_ops.causal_conv1d_shim_op (:883-902, the
                   F.pad + F.conv1d branch) and _causal_conv1d_shim_backward
                   (:910-965); the "silu" case adds F.silu + autograd on top
  fused_res.npz    kernels/hip/fused_residual_add_rmsnorm.kernel_fn_dual / kernel_fn
                   (fp32 branch, :340-391), reference.fused_residual_add_rmsnorm_ref
                   (+ autograd, plus grad_hidden for the hidden output),
                   _torch_ops._fused_res_rmsnorm_backward (:262-290) and
                   kernels/hip/fused_residual_rmsnorm_backward.kernel_fn (:265-281)
  silu_gate.npz    kernels/hip/silu_gate_mul.kernel_fn (fp32 branch, :102-110),
                   _torch_ops._silu_gate_mul_backward (:199-218),
                   kernels/hip/silu_gate_mul_backward.kernel_fn (:160-168), autograd
  rope.npz         kernels/hip/rotary_embedding.kernel_fn_fp32 (fp32 branch, :280-291),
                   reference.rotary_embedding_ref + autograd; whether
                   _torch_ops._rotary_backward (:140-162) accepts the forward's (N, D/2)
                   tables is recorded as `ref_bwd_raises`
  linear_ce.npz    F.linear + F.cross_entropy(ignore_index) fp32 + autograd, the
                   oracle of scripts/test_chunked_ce.py:13-39
The fixtures are committed; the GPU box never needs the reference.
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


class _OnCuda(torch.Tensor):
    """CPU tensor that reports is_cuda=True, so that reference entry points which
    assert CUDA (e.g. ce_full, ce_fused.py:754) run their pure-PyTorch fp32 branch
    on the CPU unchanged."""

    @property
    def is_cuda(self):  # noqa: D401
        return True


def _on_cuda(t: torch.Tensor) -> torch.Tensor:
    return torch.Tensor._make_subclass(_OnCuda, t, t.requires_grad)


class _Ctx:
    """Minimal autograd ctx stand-in for calling the reference's backward functions."""

    def __init__(self, saved, **attrs):
        self.saved_tensors = saved
        for k, v in attrs.items():
            setattr(self, k, v)


def _np(t):
    return t.detach().cpu().numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AK_REFERENCE",
                                                          str(Path(__file__).resolve().parents[3] / "reference")))
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "external" / "mamba"))
    sys.modules.setdefault("selective_scan_cuda", types.ModuleType("selective_scan_cuda"))

    import reference  # noqa: E402
    import kernels.hip._torch_ops as rops  # noqa: E402
    from kernels import ce_fused  # noqa: E402
    from models.amadeus import selective_scan_chunked  # noqa: E402
    from mamba_ssm.ops.selective_scan_interface import selective_scan_ref  # noqa: E402

    torch.set_num_threads(max(1, torch.get_num_threads()))

    # ---------------- RMSNorm (BASELINE config 0 distribution, fewer rows)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(32, 768, generator=g)
    w = 1 + 0.02 * torch.randn(768, generator=g)
    dy = torch.randn(32, 768, generator=g)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    y = reference.rmsnorm_ref(xr, wr, 1e-6)
    y.backward(dy)
    gx_fb, gw_fb = rops._rmsnorm_backward(_Ctx((x, w), eps=1e-6), dy)
    np.savez_compressed(HERE / "rmsnorm.npz", x=_np(x), w=_np(w), dy=_np(dy), eps=np.float64(1e-6),
                        y=_np(y), dx_autograd=_np(xr.grad), dw_autograd=_np(wr.grad),
                        dx_fallback=_np(gx_fb), dw_fallback=_np(gw_fb))

    # ---------------- Softmax (causal attention-score rows, config 3 distribution)
    g = torch.Generator().manual_seed(1)
    L = 128
    s = torch.randn(3, L, L, generator=g) / 8.0
    s = s.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), 1), float("-inf"))
    dys = torch.randn(3, L, L, generator=g)
    sr = s.clone().requires_grad_(True)
    ys = reference.softmax_ref(sr)
    ys.backward(dys)
    np.savez_compressed(HERE / "softmax.npz", x=_np(s), dy=_np(dys), y=_np(ys), dx=_np(sr.grad))

    # ---------------- Collapsed scan via the reference's model-side derivation
    g = torch.Generator().manual_seed(2)
    Bsz, T, d, dstate, heads = 2, 200, 48, 12, 4
    xs = torch.randn(Bsz, T, d, generator=g)
    # dt as in a Mamba dt projection (softplus(N(0,1) - 4)); the reference's chunked
    # forward divides by the in-chunk cumulative decay clamped at 1e-10
    # (models/amadeus.py:226-233), so it is only exact while that product stays
    # far above 1e-10 — which this distribution guarantees.
    dt_ = torch.nn.functional.softplus(torch.randn(Bsz, T, d, generator=g) - 4.0)
    A_log = torch.log(torch.rand(d, generator=g) * 0.9 + 0.1)
    Bm = torch.randn(Bsz, T, dstate, generator=g)
    Cm = torch.randn(Bsz, T, dstate, generator=g)
    Dv = torch.randn(d, generator=g)
    y1 = selective_scan_chunked(xs, dt_, A_log, Bm, Cm, Dv, heads)
    dA = torch.exp(dt_ * -torch.exp(A_log))
    dBx = dt_ * Bm.repeat(1, 1, heads) * xs
    Ce = Cm.repeat(1, 1, heads)
    gy = torch.randn(Bsz, T, d, generator=g)
    grads = rops._selective_scan_backward(_Ctx((dA, dBx, Ce, Dv, xs, y1)), gy)
    np.savez_compressed(HERE / "scan1.npz", dA=_np(dA), dBx=_np(dBx), C=_np(Ce), D=_np(Dv), x=_np(xs), gy=_np(gy),
                        y=_np(y1), gdA=_np(grads[0]), gdBx=_np(grads[1]), gC=_np(grads[2]), gD=_np(grads[3]),
                        gx=_np(grads[4]))

    # ---------------- Mamba-style selective scan (config 1 distribution, small shapes)
    for groups in (1, 2):
        g = torch.Generator().manual_seed(10 + groups)
        b, D_, Ls, N = 2, 8, 300, 16
        u = torch.randn(b, D_, Ls, generator=g)
        delta = torch.randn(b, D_, Ls, generator=g) - 4.6
        dtb = torch.rand(D_, generator=g) * 2 - 1
        A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D_, 1)
        shp = (b, N, Ls) if groups == 1 else (b, groups, N, Ls)
        Bv = torch.randn(*shp, generator=g)
        Cv = torch.randn(*shp, generator=g)
        Dd = torch.rand(D_, generator=g)
        z = torch.randn(b, D_, Ls, generator=g)
        dout = torch.randn(b, D_, Ls, generator=g)
        leaves = [t.clone().requires_grad_(True) for t in (u, delta, A, Bv, Cv, Dd, z, dtb)]
        out, last = selective_scan_ref(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4], D=leaves[5],
                                       z=leaves[6], delta_bias=leaves[7], delta_softplus=True,
                                       return_last_state=True)
        out.backward(dout)
        names = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]
        payload = {n: _np(t) for n, t in zip(names, (u, delta, A, Bv, Cv, Dd, z, dtb))}
        payload.update({"d" + n: _np(t.grad) for n, t in zip(names, leaves)})
        np.savez_compressed(HERE / f"sscan_g{groups}.npz", dout=_np(dout), out=_np(out), last_state=_np(last),
                            **payload)

    # ---------------- Cross entropy on logit rows (ce_full fp32 path)
    g = torch.Generator().manual_seed(3)
    Bc, V = 64, 1000
    logits = torch.randn(Bc, V, generator=g) * 3
    tg = torch.randint(0, V, (Bc,), generator=g)
    tg[::7] = -100
    cases = {"plain": dict(), "softcap": dict(softcap=5.0), "ls": dict(label_smoothing=0.1),
             "zloss": dict(z_loss_weight=1e-2), "all": dict(softcap=7.0, label_smoothing=0.05, z_loss_weight=1e-3)}
    payload = {"logits": _np(logits), "targets": _np(tg)}
    for name, kw in cases.items():
        lr = _on_cuda(logits.clone()).requires_grad_(True)
        loss = ce_fused.ce_full(lr, _on_cuda(tg), **kw)
        loss.backward()
        payload[f"{name}_loss"] = np.float64(torch.Tensor.item(loss))
        payload[f"{name}_grad"] = _np(lr.grad.as_subclass(torch.Tensor))
    np.savez_compressed(HERE / "ce.npz", **payload)

    # ---------------- Linear + CE (scripts/test_chunked_ce.py:13-39 reference)
    g = torch.Generator().manual_seed(4)
    Nt, Dh, Vv = 96, 64, 1000
    H = torch.randn(Nt, Dh, generator=g)
    W = torch.randn(Vv, Dh, generator=g) * 0.02 * 8
    lab = torch.randint(0, Vv, (Nt,), generator=g)
    lab[::20] = -100
    Hr = H.clone().requires_grad_(True)
    Wr = W.clone().requires_grad_(True)
    lossl = torch.nn.functional.cross_entropy(torch.nn.functional.linear(Hr, Wr), lab, ignore_index=-100)
    lossl.backward()
    np.savez_compressed(HERE / "linear_ce.npz", H=_np(H), W=_np(W), labels=_np(lab), loss=np.float64(lossl.item()),
                        dH=_np(Hr.grad), dW=_np(Wr.grad))
    # ---------------- fused residual add + RMSNorm (fp32 branches of the reference)
    from kernels.hip import fused_residual_add_rmsnorm as rfra
    from kernels.hip import fused_residual_rmsnorm_backward as rfrb
    g = torch.Generator().manual_seed(6)
    xa = torch.randn(24, 768, generator=g)
    ra = torch.randn(24, 768, generator=g)
    wa = 1 + 0.1 * torch.randn(768, generator=g)
    gha = torch.randn(24, 768, generator=g)
    gna = torch.randn(24, 768, generator=g)
    hid, nrm = rfra.kernel_fn_dual(_on_cuda(xa), _on_cuda(ra), _on_cuda(wa))
    single = rfra.kernel_fn(_on_cuda(xa), _on_cuda(ra), _on_cuda(wa))
    ref_fn = reference.fused_residual_add_rmsnorm_ref(xa, ra, wa)
    gx, gr, gw = rops._fused_res_rmsnorm_backward(_Ctx((hid.as_subclass(torch.Tensor), wa), eps=1e-6), gha, gna)
    bx, br, bw = rfrb.kernel_fn(_on_cuda(hid.as_subclass(torch.Tensor)), _on_cuda(wa), _on_cuda(gha), _on_cuda(gna))
    xg, rg, wg = (t.clone().requires_grad_(True) for t in (xa, ra, wa))
    reference.fused_residual_add_rmsnorm_ref(xg, rg, wg).backward(gna)
    np.savez_compressed(HERE / "fused_res.npz", x=_np(xa), residual=_np(ra), w=_np(wa), grad_hidden=_np(gha),
                        dx_autograd=_np(xg.grad + gha), dres_autograd=_np(rg.grad + gha), dw_autograd=_np(wg.grad),
                        grad_normed=_np(gna), hidden=_np(hid), normed=_np(nrm), single=_np(single),
                        ref_fn=_np(ref_fn), dx_op=_np(gx), dres_op=_np(gr), dw_op=_np(gw), dx_kfn=_np(bx),
                        dres_kfn=_np(br), dw_kfn=_np(bw))

    # ---------------- SiLU gate multiply (fp32 branches of the reference)
    from kernels.hip import silu_gate_mul as rsg
    from kernels.hip import silu_gate_mul_backward as rsgb
    g = torch.Generator().manual_seed(7)
    gs_ = 3 * torch.randn(64, 520, generator=g)
    us_ = torch.randn(64, 520, generator=g)
    dys = torch.randn(64, 520, generator=g)
    ysg = rsg.kernel_fn(_on_cuda(gs_), _on_cuda(us_))
    dg_op, du_op = rops._silu_gate_mul_backward(_Ctx((gs_, us_)), dys)
    dg_k, du_k = rsgb.kernel_fn(_on_cuda(gs_), _on_cuda(us_), _on_cuda(dys))
    ga, ua = gs_.clone().requires_grad_(True), us_.clone().requires_grad_(True)
    (torch.nn.functional.silu(ga) * ua).backward(dys)
    np.savez_compressed(HERE / "silu_gate.npz", gate=_np(gs_), up=_np(us_), dy=_np(dys), y=_np(ysg),
                        dgate_op=_np(dg_op), dup_op=_np(du_op), dgate_kfn=_np(dg_k), dup_kfn=_np(du_k),
                        dgate_autograd=_np(ga.grad), dup_autograd=_np(ua.grad))

    # ---------------- rotary embedding (interleaved pairs)
    from kernels.hip import rotary_embedding as rre
    g = torch.Generator().manual_seed(8)
    Bq, Hq, Nq, Dq = 2, 3, 40, 64
    xq = torch.randn(Bq, Hq, Nq, Dq, generator=g)
    inv = 1.0 / (10000.0 ** (torch.arange(0, Dq, 2, dtype=torch.float32) / Dq))
    ang = torch.outer(torch.arange(Nq, dtype=torch.float32), inv)
    cq, sq = ang.cos(), ang.sin()
    dyq = torch.randn(Bq, Hq, Nq, Dq, generator=g)
    yq = rre.kernel_fn_fp32(_on_cuda(xq), cq, sq)
    xr = xq.clone().requires_grad_(True)
    reference.rotary_embedding_ref(xr, cq, sq).backward(dyq)
    try:
        rops._rotary_backward(_Ctx((cq, sq), x_dtype=torch.float32), dyq)
        raises = False
    except RuntimeError:
        raises = True
    np.savez_compressed(HERE / "rope.npz", x=_np(xq), cos=_np(cq), sin=_np(sq), dy=_np(dyq), y=_np(yq),
                        y_ref=_np(reference.rotary_embedding_ref(xq, cq, sq)), dx_autograd=_np(xr.grad),
                        ref_bwd_raises=np.bool_(raises))

    # ---------------- causal conv1d (reference op; T crosses the 256-step kernel chunk)
    g = torch.Generator().manual_seed(5)
    payload = {}
    for tag, (B, D, T, K) in {"k4": (2, 16, 300, 4), "k3": (2, 8, 37, 3)}.items():
        xc = torch.randn(B, D, T, generator=g)
        wc = 0.5 * torch.randn(D, K, generator=g)
        bc = 0.1 * torch.randn(D, generator=g)
        dyc = torch.randn(B, D, T, generator=g)
        yc = rops.causal_conv1d_shim_op(xc, wc, bc)
        gxc, gwc, gbc = rops._causal_conv1d_shim_backward(_Ctx((xc, wc, bc)), dyc)
        xs, ws, bs = (t.clone().requires_grad_(True) for t in (xc, wc, bc))
        with torch.enable_grad():
            ys = torch.nn.functional.silu(rops.causal_conv1d_shim_op(xs, ws, bs))
            ys.backward(dyc)
        payload.update({f"{tag}_x": _np(xc), f"{tag}_w": _np(wc), f"{tag}_b": _np(bc), f"{tag}_dy": _np(dyc),
                        f"{tag}_y": _np(yc), f"{tag}_dx": _np(gxc), f"{tag}_dw": _np(gwc), f"{tag}_db": _np(gbc),
                        f"{tag}_silu_y": _np(ys), f"{tag}_silu_dx": _np(xs.grad), f"{tag}_silu_dw": _np(ws.grad),
                        f"{tag}_silu_db": _np(bs.grad)})
    np.savez_compressed(HERE / "conv1d.npz", **payload)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
