"""Benchmark of the hot path on B200: selective-scan forward+backward (headline)
plus the other swapped ops, with roofline fractions and a CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Headline workload: Mamba-style selective scan, B=8,
D=1536, L=2048, N=16, bf16 inputs, fp32 state, softplus(delta + bias), SiLU(z)
gate, last state; one step = forward + backward over one batch per rank
(weak scaling: every rank processes its own batch; no collective on the data
path).  `value` = algorithmic bytes of all ranks / max-over-ranks device time.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "autokernel-halo-strix_b200"
for _p in (str(PKG), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

HEADLINE = dict(batch=8, dim=1536, L=2048, N=16, groups=1)
METRIC = "selective_scan fwd+bwd HBM GB/s (algorithmic bytes / device time)"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# dram__bytes_read.sum + dram__bytes_write.sum per launch from ncu captures, scaled
# to the full config where the capture was smaller (see profiles/).  None = not captured.
NCU_TRAFFIC_BYTES = {
    # B=4 capture (profiles/selective_scan_kernels_B4_*): 106,179,072 read + 42,633,984 written,
    # x2 for B=8 (every input, output and B/C tile is per batch row, so traffic is linear in B)
    "sscan_bwd": 2 * (106_179_072 + 42_633_984),
}
# smsp__inst_executed.sum (warp-instructions) per launch of the scan backward at the headline
# shape, from the same kind of capture (B=4, doubled: the instruction count is linear in B) of
# the current kernel (paired fp32 step pairs; profiles/selective_scan_kernels_B4_*, instruction
# mix by opcode: 303.9 M at B=4, 48.3 per (step, state) lane-unit).
# The backward is issue-bound, so its roofline is the SM's issue rate: 148 SMs x 4 schedulers x
# one warp-instruction per clock at the clock sampled during the timed region.
NCU_WARP_INST = {
    "sscan_bwd": 2 * 303_900_000,
}


# ----------------------------------------------------------------------------
# algorithmic bytes
# ----------------------------------------------------------------------------
def sscan_bytes(batch, dim, L, N, groups, es=2):
    E = batch * dim * L
    bc = batch * groups * N * L * es
    par = dim * N * 4 + 2 * dim * 4
    fwd = 3 * E * es + 2 * bc + par + E * es + batch * dim * N * 4
    bwd = 4 * E * es + 2 * bc + par + 3 * E * es + 2 * bc + dim * N * 4 + 2 * dim * 4
    return fwd, bwd


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


# ----------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ----------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# distributed helpers
# ----------------------------------------------------------------------------
def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"  # keep stdout to the one JSON line
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------
# workloads
# ----------------------------------------------------------------------------
def make_sscan_inputs(cfg, dev, seed, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    b, dim, L, N = cfg["batch"], cfg["dim"], cfg["L"], cfg["N"]
    import math
    dt_min, dt_max = 1e-3, 1e-1
    dtv = torch.exp(torch.rand(dim, generator=g) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
    dtv = dtv.clamp(min=1e-4)
    inv_dt = dtv + torch.log(-torch.expm1(-dtv))  # mamba_simple.py:91-99 dt-bias init
    host = dict(
        u=torch.randn(b, dim, L, generator=g).to(dtype),
        delta=(torch.randn(b, dim, L, generator=g) - 4.6).to(dtype),
        A=-torch.arange(1, N + 1, dtype=torch.float32).repeat(dim, 1),
        B=torch.randn(b, N, L, generator=g).to(dtype),
        C=torch.randn(b, N, L, generator=g).to(dtype),
        D=torch.rand(dim, generator=g),
        z=torch.randn(b, dim, L, generator=g).to(dtype),
        delta_bias=inv_dt.float(),
        dout=torch.randn(b, dim, L, generator=g).to(dtype),
    )
    return host


def time_sscan(cfg, dev, steps, warmup, world):
    from kernels import _ak
    host = make_sscan_inputs(cfg, dev, seed=1234 + (dist.get_rank() if world > 1 else 0))
    d = {k: v.to(dev) for k, v in host.items()}
    st = torch.cuda.current_stream(dev)

    def step(ev=None):
        if ev:
            ev[0].record(st)
        out, last, states = _ak.selective_scan_fwd(d["u"], d["delta"], d["A"], d["B"], d["C"], d["D"], d["z"],
                                                   d["delta_bias"], True)
        if ev:
            ev[1].record(st)
        grads = _ak.selective_scan_bwd(d["dout"], d["u"], d["delta"], d["A"], d["B"], d["C"], d["D"], d["z"],
                                       d["delta_bias"], True, states)
        if ev:
            ev[2].record(st)
        return out, grads

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        start.record(st)
        for i in range(steps):
            step(evs[i])
        end.record(st)
        torch.cuda.synchronize(dev)
    barrier(world)
    total_ms = start.elapsed_time(end)
    fwd_ms = [e[0].elapsed_time(e[1]) for e in evs]
    bwd_ms = [e[1].elapsed_time(e[2]) for e in evs]
    return total_ms, fwd_ms, bwd_ms, clk.summary(), host


def time_comparator(dev, host, steps, warmup, our_fwd_ms, our_bwd_ms):
    """The reference's own GPU kernel for the headline scan (mamba_ssm 2.3.0 `selective_scan_cuda`,
    built for sm_100a from the reference sources into oracle/_ref/ by oracle/build_mamba_ref.py),
    timed in this process on the same inputs with the same CUDA-event protocol as ours.  It is a
    reference arm, not our measurement; None when the module was not built."""
    try:
        from oracle.build_mamba_ref import load_built
        mod = load_built()
    except Exception as e:  # noqa: BLE001 - a missing comparator never stops the bench
        return {"unavailable": f"comparator failed to load: {e}"[:200]}
    if mod is None:
        return {"unavailable": "reference selective_scan_cuda not built (needs the reference checkout)"}
    d = {k: v.to(dev) for k, v in host.items()}
    B4, C4 = d["B"].unsqueeze(1), d["C"].unsqueeze(1)
    st = torch.cuda.current_stream(dev)

    def fwd():
        return mod.fwd(d["u"], d["delta"], d["A"], B4, C4, d["D"], d["z"], d["delta_bias"], True)

    def bwd(r):
        out, x, _ = r
        mod.bwd(d["u"], d["delta"], d["A"], B4, C4, d["D"], d["z"], d["delta_bias"], d["dout"], x, out, None,
                True, False)

    for _ in range(warmup):
        bwd(fwd())
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for e in evs:
        e[0].record(st)
        r = fwd()
        e[1].record(st)
        bwd(r)
        e[2].record(st)
    torch.cuda.synchronize(dev)
    rf = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    rb = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    del d
    torch.cuda.empty_cache()
    return {"impl": "mamba_ssm 2.3.0 selective_scan_cuda (reference sources, built for sm_100a)",
            "fwd_ms": round(rf, 4), "bwd_ms": round(rb, 4), "total_ms": round(rf + rb, 4),
            "ours_total_ms": round(our_fwd_ms + our_bwd_ms, 4),
            "speedup_fwd": round(rf / our_fwd_ms, 3), "speedup_bwd": round(rb / our_bwd_ms, 3),
            "speedup_total": round((rf + rb) / (our_fwd_ms + our_bwd_ms), 3)}


def time_sscan_e2e(cfg, dev, steps, warmup, host, slices=8):
    """Same step through the public API (selective_scan_fn + autograd) with inputs in pinned
    host memory: every step copies all its inputs H2D and reads a result (last_state) back D2H.

    The batch rows are independent, so the step is pipelined over `slices` batch slices: slice
    i+1 is copied on a copy stream while slice i runs fwd+bwd on the compute stream.  A, D and
    delta_bias are shared leaves, so their gradients accumulate to the full-batch values exactly as
    in one call.  Device buffers are allocated once, outside the timed region; the copies are
    inside it (the copy stream waits on the start event)."""
    from kernels.mamba_scan import selective_scan_fn
    b = cfg["batch"]
    slices = slices if b % slices == 0 else 1
    rows = b // slices
    pinned = {k: v.pin_memory() for k, v in host.items()}
    h2d = sum(v.numel() * v.element_size() for v in pinned.values())
    res_host = torch.empty(b, cfg["dim"], cfg["N"], dtype=torch.float32).pin_memory()
    st = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    shared = ("A", "D", "delta_bias")
    per_row = [k for k in pinned if k not in shared]
    dev_sh = {k: torch.empty_like(pinned[k], device=dev) for k in shared}
    dev_sl = [{k: torch.empty_like(pinned[k][i * rows:(i + 1) * rows], device=dev) for k in per_row}
              for i in range(slices)]
    copied = [torch.cuda.Event() for _ in range(slices + 1)]
    used = [torch.cuda.Event() for _ in range(slices + 1)]
    for ev in used:
        ev.record(st)

    def step(start_ev):
        with torch.cuda.stream(cs):
            cs.wait_event(start_ev)
            cs.wait_event(used[slices])
            for k in shared:
                dev_sh[k].copy_(pinned[k], non_blocking=True)
            copied[slices].record(cs)
            for i in range(slices):
                cs.wait_event(used[i])  # the previous step is done with this slice's buffers
                for k in per_row:
                    dev_sl[i][k].copy_(pinned[k][i * rows:(i + 1) * rows], non_blocking=True)
                copied[i].record(cs)
        st.wait_event(copied[slices])
        sh = {k: v.detach().requires_grad_(True) for k, v in dev_sh.items()}
        for i in range(slices):
            st.wait_event(copied[i])
            d = dev_sl[i]
            leaves = [d[k].detach().requires_grad_(True) for k in ("u", "delta")]
            Bm, Cm, z = (d[k].detach().requires_grad_(True) for k in ("B", "C", "z"))
            out, last = selective_scan_fn(leaves[0], leaves[1], sh["A"], Bm, Cm, D=sh["D"], z=z,
                                          delta_bias=sh["delta_bias"], delta_softplus=True,
                                          return_last_state=True)
            out.backward(d["dout"])
            res_host[i * rows:(i + 1) * rows].copy_(last, non_blocking=True)
            used[i].record(st)
        used[slices].record(st)
        return res_host

    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(warmup):
        w = torch.cuda.Event()
        w.record(st)
        step(w)
    torch.cuda.synchronize(dev)
    s.record(st)
    for _ in range(steps):
        step(s)
    e.record(st)
    torch.cuda.synchronize(dev)
    step_ms = s.elapsed_time(e) / steps
    # the step's copy bound: the same H2D copies alone, back to back on the copy stream
    cs_s, cs_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cs):
        for rep in range(warmup + steps):
            if rep == warmup:
                cs_s.record(cs)
            for k in shared:
                dev_sh[k].copy_(pinned[k], non_blocking=True)
            for i in range(slices):
                for k in per_row:
                    dev_sl[i][k].copy_(pinned[k][i * rows:(i + 1) * rows], non_blocking=True)
        cs_e.record(cs)
    torch.cuda.synchronize(dev)
    copy_ms = cs_s.elapsed_time(cs_e) / steps
    d2h = res_host.numel() * res_host.element_size()
    return step_ms, h2d, d2h, copy_ms


def cpu_sscan_sample(dim_sample=48, L=2048, N=16, repeats=1):
    """Oracle (the reference's selective_scan_ref restated, fp32 on the host cores) timed on a
    bounded sample: batch 1, `dim_sample` channels, full L, fwd + autograd bwd."""
    from oracle import hot_path_oracle as O
    cfg = dict(batch=1, dim=dim_sample, L=L, N=N, groups=1)
    host = make_sscan_inputs(cfg, None, seed=7, dtype=torch.float32)
    t0 = time.perf_counter()
    for _ in range(repeats):
        O.selective_scan_grads(host["u"], host["delta"], host["A"], host["B"], host["C"], host["D"], host["z"],
                               host["delta_bias"], True, host["dout"], dt=torch.float32)
    dt = (time.perf_counter() - t0) / repeats
    fwd, bwd = sscan_bytes(1, dim_sample, L, N, 1, es=2)
    return {"value": round((fwd + bwd) / dt / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"batch 1 x {dim_sample} channels x L={L} x N={N}, fp32 fwd+bwd (oracle restatement of "
                      f"selective_scan_ref + autograd), {dt:.2f} s/step; GB/s counts the bf16 algorithmic bytes "
                      f"of the same sample"}


def cpu_ops_sample():
    """The reference's CPU path for the other rows (restated in `oracle/`, fp32 on the host cores),
    each on a bounded sample of its BASELINE config; same units as the GPU `ops` lines (GB/s of
    algorithmic bytes, TFLOP/s for linear+CE), forward + backward per sample."""
    from oracle import hot_path_oracle as O
    f32 = torch.float32
    g = torch.Generator().manual_seed(11)
    res = {}

    def timed(fn, reps=2):
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    # RMSNorm fp32 [8192, 768] (full config): fwd + bwd, 125.8 MB algorithmic
    x = torch.randn(8192, 768, generator=g)
    w = 1 + 0.02 * torch.randn(768, generator=g)
    dy = torch.randn(8192, 768, generator=g)
    t = timed(lambda: (O.rmsnorm_fwd(x, w, dt=f32), O.rmsnorm_bwd(x, w, dy, dt=f32)))
    res["rmsnorm_fwd_bwd_fp32_8192x768"] = {"GB/s": round(125_838_336 / t / 1e9, 3), "s": round(t, 4),
                                            "sample": "full config"}
    # softmax: 2048 of the 196608 rows x 2048 (fp32 math on bf16-valued data), fwd + bwd = 5 row passes
    sx = (torch.randn(2048, 2048, generator=g) / 8).to(torch.bfloat16).float()
    sdy = torch.randn(2048, 2048, generator=g)
    t = timed(lambda: O.softmax_bwd(O.softmax_fwd(sx, dt=f32), sdy, dt=f32))
    res["softmax_fwd_bwd_bf16_2048x2048_sample"] = {"GB/s": round(5 * 2048 * 2048 * 2 / t / 1e9, 3),
                                                    "s": round(t, 4), "sample": "2048 of 196608 rows"}
    # collapsed scan: 1 of 8 batch rows, (1, 2048, 1536) fp32, fwd + bwd = 56 B/elt
    dA = torch.rand(1, 2048, 1536, generator=g) * 0.5 + 0.5
    dBx, Cm, xs, gy = (torch.randn(1, 2048, 1536, generator=g) for _ in range(4))
    Dv = torch.randn(1536, generator=g)
    t = timed(lambda: O.scan1_bwd(dA, dBx, Cm, Dv, xs, gy, dt=f32), reps=1)
    res["scan1_fwd_bwd_fp32_1x2048x1536_sample"] = {"GB/s": round(56 * 2048 * 1536 / t / 1e9, 3),
                                                    "s": round(t, 4), "sample": "batch 1 of 8"}
    # linear + CE: 512 of the 32768 rows, D 768, V 50304, fp32 GEMMs + CE + autograd (3 * 2NDV FLOP)
    H = torch.randn(512, 768, generator=g)
    Wt = torch.randn(50304, 768, generator=g) * 0.02
    lab = torch.randint(0, 50257, (512,), generator=g)
    t = timed(lambda: O.linear_ce(H, Wt, lab, dt=f32), reps=1)
    res["linear_ce_fp32_512x768x50304_sample"] = {"TFLOP/s": round(6 * 512 * 768 * 50304 / t / 1e12, 4),
                                                  "s": round(t, 4), "sample": "512 of 32768 rows"}
    # SiLU-gate, fused residual RMSNorm, RoPE, causal conv1d: 1/16 samples of their GPU cases
    gt, up, gd = (torch.randn(4096, 2048, generator=g) for _ in range(3))
    t = timed(lambda: (O.silu_gate_mul(gt, up, dt=f32), O.silu_gate_mul_bwd(gt, up, gd, dt=f32)))
    res["silu_gate_fwd_bwd_4096x2048_sample"] = {"GB/s": round(8 * 4096 * 2048 * 2 / t / 1e9, 3),
                                                 "s": round(t, 4), "sample": "4096 of 65536 rows"}
    xr, rr, gh, gn = (torch.randn(4096, 768, generator=g) for _ in range(4))
    t = timed(lambda: (O.fused_res_rmsnorm(xr, rr, w, dt=f32),
                       O.fused_res_rmsnorm_bwd(xr + rr, w, gh, gn, dt=f32)))
    res["fused_res_rmsnorm_fwd_bwd_4096x768_sample"] = {"GB/s": round(8 * 4096 * 768 * 2 / t / 1e9, 3),
                                                        "s": round(t, 4), "sample": "4096 of 65536 rows"}
    q = torch.randn(4, 12, 2048, 64, generator=g)
    ang = torch.outer(torch.arange(2048, dtype=f32), 1.0 / (10000.0 ** (torch.arange(0, 64, 2, dtype=f32) / 64)))
    t = timed(lambda: (O.rope(q, ang.cos(), ang.sin(), dt=f32), O.rope_bwd(q, ang.cos(), ang.sin(), dt=f32)))
    res["rope_fwd_bwd_4x12x2048x64_sample"] = {"GB/s": round(4 * q.numel() * 2 / t / 1e9, 3), "s": round(t, 4),
                                               "sample": "batch 4 of 64"}
    xc, dc = (torch.randn(1, 1536, 2048, generator=g) for _ in range(2))
    wc, bc = torch.randn(1536, 4, generator=g), torch.randn(1536, generator=g)
    t = timed(lambda: O.causal_conv1d_grads(xc, wc, bc, dc, silu=True, dt=f32))
    res["conv1d_silu_fwd_bwd_1x1536x2048_sample"] = {"GB/s": round(5 * xc.numel() * 2 / t / 1e9, 3),
                                                     "s": round(t, 4), "sample": "batch 1 of 16"}
    return {"cores": torch.get_num_threads(), "kind": "port", "ops": res}


def time_other_ops(dev, steps, warmup, hbm_peak, bf16_peak, which=None, ce_rows=32768, scale=1):
    """Device-timed throughput of the other swapped ops at their BASELINE configs.
    `which`: subset of {"rmsnorm", "softmax", "linear_ce", "scan1", "ce_rows", "fused_res", "silu_gate", "rope", "conv1d"} (None = all)."""
    from kernels import _ak
    res = {}
    st = torch.cuda.current_stream(dev)

    def want(name):
        return which is None or name in which

    def timeit(fn, nbytes, name, reps, graph=False):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        run = fn
        if graph:
            # short kernels: replay the calls from a CUDA graph so host-side argument
            # marshalling does not starve the GPU; the graph holds exactly the launches
            # one call makes
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            run = gr.replay
            run()
            torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(reps):
            run()
        b.record(st)
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b) / reps
        gbs = nbytes / ms / 1e6
        res[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac": round(gbs / hbm_peak, 3)}

    if want("rmsnorm"):
        # RMSNorm fp32 [8192, 768] (config 0): 25 MB per tensor < L2, so a 256 MB scratch
        # write flushes L2 before each repetition and its own time is subtracted.
        g = torch.Generator().manual_seed(0)
        x = torch.randn(8192, 768, generator=g).to(dev)
        w = (1 + 0.02 * torch.randn(768, generator=g)).to(dev)
        dy = torch.randn(8192, 768, generator=g).to(dev)
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        E = 8192 * 768
        fw_b, bw_b = 2 * E * 4 + 768 * 4, 3 * E * 4 + 2 * 768 * 4
        timeit(lambda: flush.zero_(), 1, "_flush", steps * 4)
        fl = res.pop("_flush")["ms"]
        timeit(lambda: (flush.zero_(), _ak.rmsnorm_fwd(x, w, 1e-6)), fw_b, "rmsnorm_fwd_fp32_8192x768", steps * 4)
        timeit(lambda: (flush.zero_(), _ak.rmsnorm_bwd(x, w, dy, 1e-6)), bw_b, "rmsnorm_bwd_fp32_8192x768", steps * 4)
        # size ceiling: a plain torch copy of one such tensor (25 MB in, 25 MB out) under the same protocol
        ycp = torch.empty_like(x)
        timeit(lambda: (flush.zero_(), ycp.copy_(x)), 2 * E * 4, "_copy32", steps * 4)
        cp32 = 2 * E * 4 / max(res.pop("_copy32")["ms"] - fl, 1e-6) / 1e6 / hbm_peak
        for k, nb in (("rmsnorm_fwd_fp32_8192x768", fw_b), ("rmsnorm_bwd_fp32_8192x768", bw_b)):
            ms = max(res[k]["ms"] - fl, 1e-6)
            gbs = nb / ms / 1e6
            res[k] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac": round(gbs / hbm_peak, 3),
                      "copy_ceiling_frac": round(cp32, 3),
                      "note": "L2 flushed (256 MB write) before each rep; flush time subtracted; "
                              "copy_ceiling_frac = a plain 25 MB -> 25 MB copy under the same protocol"}
        del x, dy, ycp, flush
        # bf16 at the training shape [16384, 768] (16 x 1024 tokens per GPU): 25 MB per tensor, same flush
        xb = torch.randn(16384, 768, generator=g).to(torch.bfloat16).to(dev)
        wb = (1 + 0.02 * torch.randn(768, generator=g)).to(torch.bfloat16).to(dev)
        dyb = torch.randn(16384, 768, generator=g).to(torch.bfloat16).to(dev)
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        Eb = 16384 * 768
        fwb, bwb = 2 * Eb * 2 + 768 * 2, 3 * Eb * 2 + 2 * 768 * 2
        timeit(lambda: (flush.zero_(), _ak.rmsnorm_fwd(xb, wb, 1e-6)), fwb, "rmsnorm_fwd_bf16_16384x768", steps * 4)
        timeit(lambda: (flush.zero_(), _ak.rmsnorm_bwd(xb, wb, dyb, 1e-6)), bwb, "rmsnorm_bwd_bf16_16384x768",
               steps * 4)
        ycp = torch.empty_like(xb)
        timeit(lambda: (flush.zero_(), ycp.copy_(xb)), 2 * Eb * 2, "_copy16", steps * 4)
        cp16 = 2 * Eb * 2 / max(res.pop("_copy16")["ms"] - fl, 1e-6) / 1e6 / hbm_peak
        del ycp
        for k, nb in (("rmsnorm_fwd_bf16_16384x768", fwb), ("rmsnorm_bwd_bf16_16384x768", bwb)):
            ms = max(res[k]["ms"] - fl, 1e-6)
            gbs = nb / ms / 1e6
            res[k] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac": round(gbs / hbm_peak, 3),
                      "copy_ceiling_frac": round(cp16, 3),
                      "note": "L2 flushed (256 MB write) before each rep; flush time subtracted; "
                              "copy_ceiling_frac = a plain 25 MB -> 25 MB copy under the same protocol"}
        del xb, dyb, flush
        # Second protocol, no flush: one CUDA graph of 16 calls, each on its own buffers (16 sets
        # of 50-75 MB rotate through > 1 GB, so every call reads from HBM); time = replay / 16.
        torch.cuda.empty_cache()
        for dt, rows in ((torch.float32, 8192), (torch.bfloat16, 16384)):
            sets = [(torch.randn(rows, 768, device=dev).to(dt), torch.randn(rows, 768, device=dev).to(dt))
                    for _ in range(16)]
            wr = (1 + 0.02 * torch.randn(768, device=dev)).to(dt)
            es = 2 if dt == torch.bfloat16 else 4
            E = rows * 768
            tag = f"{'bf16' if es == 2 else 'fp32'}_{rows}x768"
            for name, nb, fn in (("fwd", 2 * E * es + 768 * es, lambda x, d: _ak.rmsnorm_fwd(x, wr, 1e-6)),
                                 ("bwd", 3 * E * es + 2 * 768 * es, lambda x, d: _ak.rmsnorm_bwd(x, wr, d, 1e-6))):
                def calls(fn=fn):
                    for x, d in sets:
                        fn(x, d)
                timeit(calls, 16 * nb, "x", max(3, steps // 2), graph=True)
                r = res.pop("x")
                key = f"rmsnorm_{name}_{tag}"
                res[key]["rotating_buffers"] = {"ms": round(r["ms"] / 16, 4), "GB/s": r["GB/s"], "frac": r["frac"],
                                                "note": "16 calls on 16 buffer sets in one CUDA graph, no flush"}
            del sets
            torch.cuda.empty_cache()

    if want("softmax"):
        # Softmax causal scores bf16 [96*2048, 2048] (config 3): 805 MB per tensor > L2.
        rows, cols = 96 * 2048 // scale, 2048
        s = (torch.randn(rows, cols, device=dev) / 8).to(torch.bfloat16)
        r = torch.arange(rows, device=dev) % cols
        s.masked_fill_(torch.arange(cols, device=dev)[None, :] > r[:, None], float("-inf"))
        dys = torch.randn(rows, cols, device=dev).to(torch.bfloat16)
        y = _ak.softmax_fwd(s)
        T = rows * cols * 2
        timeit(lambda: _ak.softmax_fwd(s), 2 * T, "softmax_fwd_bf16_196608x2048", steps)
        timeit(lambda: _ak.softmax_bwd(y, dys), 3 * T, "softmax_bwd_bf16_196608x2048", steps)
        del s, dys, y

    if want("linear_ce"):
        # Fused linear + CE (config 2): H [32768, 768], W [50304, 768] bf16, 5% ignored.
        # Algorithmic FLOPs 3 * 2NDV (logits, dH, dW).
        Nt, Dh, Vv = ce_rows, 768, 50304
        g = torch.Generator().manual_seed(0)
        H = torch.randn(Nt, Dh, generator=g).to(torch.bfloat16).to(dev)
        W = (torch.randn(Vv, Dh, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        lab = torch.randint(0, 50257, (Nt,), generator=g)
        lab[torch.randperm(Nt, generator=g)[: Nt // 20]] = -100
        lab = lab.to(dev)
        flops = 3 * 2 * Nt * Dh * Vv
        tag = f"bf16_{Nt}x{Dh}x{Vv}"
        from kernels.hip.chunked_linear_cross_entropy import _ChunkedLinearCrossEntropy, _FusedLinearCrossEntropy
        timeit(lambda: _FusedLinearCrossEntropy.apply(H.requires_grad_(True), W.requires_grad_(True), lab, -100), 1,
               "linear_ce_module", max(2, steps // 4))
        ms3 = res.pop("linear_ce_module")["ms"]
        tf3 = flops / (ms3 / 1e3) / 1e12
        res[f"linear_ce_{tag}"] = {
            "ms": ms3, "TFLOP/s": round(tf3, 1), "frac_bf16": round(tf3 / bf16_peak, 3),
            "note": "ChunkedLinearCrossEntropyLoss path (_FusedLinearCrossEntropy -> ak_linear_ce_fwdbwd): "
                    "logits, dW and dH on our 2-SM tcgen05 GEMM, statistics epilogue, in-place dlogits; "
                    "algorithmic 3*2NDV"}
        timeit(lambda: _ak.linear_ce_fwdbwd(H, W, lab, -100), 1, "x", max(2, steps // 4))
        ms = res.pop("x")["ms"]
        tf = flops / (ms / 1e3) / 1e12
        res[f"linear_ce_all_tcgen05_{tag}"] = {
            "ms": ms, "TFLOP/s": round(tf, 1), "frac_bf16": round(tf / bf16_peak, 3),
            "note": "ak_linear_ce_fwdbwd through the C-ABI wrapper directly (no autograd), same kernels"}
        timeit(lambda: _ChunkedLinearCrossEntropy.apply(H.requires_grad_(True), W.requires_grad_(True), lab, 4096,
                                                        0.0, -100, 0.0, 0.0), 1, "x", 2)
        ms2 = res.pop("x")["ms"]
        res[f"linear_ce_chunked_cublas_{tag}"] = {
            "ms": ms2, "TFLOP/s": round(flops / (ms2 / 1e3) / 1e12, 1),
            "note": "library comparator: cuBLAS GEMMs around the CE row kernel, 4096-row chunks"}
        # our tcgen05 GEMM against cuBLAS on the three contractions of one 16384-row chunk
        Nc = min(16384, Nt)
        G = (torch.randn(Nc, Vv, device=dev) * 1e-3).to(torch.bfloat16)
        Hc = H[:Nc]
        cmp = {}
        for name, ours, lib, fl in (
                ("logits", lambda: _ak.tc_gemm(Hc, W.t()), lambda: torch.mm(Hc, W.t()), 2 * Nc * Vv * Dh),
                ("dW", lambda: _ak.tc_gemm(G.t(), Hc, out_dtype=torch.float32),
                 lambda: torch.mm(G.t(), Hc, out_dtype=torch.float32), 2 * Vv * Dh * Nc),
                ("dH", lambda: _ak.tc_gemm(G, W), lambda: torch.mm(G, W), 2 * Nc * Dh * Vv)):
            timeit(ours, 1, "x", max(3, steps // 4))
            mo = res.pop("x")["ms"]
            timeit(lib, 1, "x", max(3, steps // 4))
            ml = res.pop("x")["ms"]
            cmp[name] = {"ours_ms": mo, "cublas_ms": ml, "ours_TFLOP/s": round(fl / (mo / 1e3) / 1e12, 1),
                         "ratio_vs_cublas": round(ml / mo, 3)}
        res[f"linear_ce_gemms_vs_cublas_{Nc}x{Dh}x{Vv}"] = cmp
        del H, W, lab, G, Hc
        torch.cuda.empty_cache()

    if want("scan1"):
        # Collapsed scan fp32 (8, 2048, 1536): 100 MB per tensor.
        Bsz, L, d = 8, 2048, 1536
        dA = torch.rand(Bsz, L, d, device=dev) * 0.5 + 0.5
        dBx, C, xx, gy = (torch.randn(Bsz, L, d, device=dev) for _ in range(4))
        Dv = torch.randn(d, device=dev)
        E = Bsz * L * d
        # the product path (autokernel::selective_scan): the forward saves the 64-step chunk-start
        # states (B * L/64 * d floats) and the backward reuses them
        timeit(lambda: _ak.scan1_fwd(dA, dBx, C, Dv, xx, save_carries=True), 20 * E, "scan1_fwd_fp32_8x2048x1536",
               steps)
        _y, carries = _ak.scan1_fwd(dA, dBx, C, Dv, xx, save_carries=True)
        timeit(lambda: _ak.scan1_bwd(dA, dBx, C, Dv, xx, gy, carries=carries), 36 * E, "scan1_bwd_fp32_8x2048x1536",
               steps)
        # the reference-shaped C entry without saved states (re-derives them: +8 bytes per element)
        timeit(lambda: _ak.scan1_bwd(dA, dBx, C, Dv, xx, gy), 36 * E, "scan1_bwd_nocarries_fp32_8x2048x1536", steps)
        del dA, dBx, C, xx, gy, _y, carries
        torch.cuda.empty_cache()

    if want("ce_rows"):
        # CE rows with fused gradient, bf16 logits [4096, 50304] (one chunk of the chunked linear+CE
        # path; 412 MB): reads each row once for the statistics, once more (L2) for the gradient,
        # writes the gradient.  Algorithmic bytes: logits read + gradient written.
        Nc, Vc = 4096 // scale if scale > 1 else 4096, 50304
        lg = (torch.randn(Nc, Vc, device=dev) * 2).to(torch.bfloat16)
        tg = torch.randint(0, Vc, (Nc,), device=dev)
        E = Nc * Vc
        timeit(lambda: _ak.ce_rows_fwd(lg, tg, write_grad=True), 4 * E, "ce_rows_fwd_grad_bf16_4096x50304", steps,
               graph=True)
        del lg, tg
        torch.cuda.empty_cache()

    if want("fused_res"):
        # Fused residual add + RMSNorm bf16 [65536, 768] (the hybrid's d_model; 100 MB per tensor):
        # fwd reads x, residual and writes hidden, normed; bwd reads hidden, grad_hidden,
        # grad_normed and writes dx.
        Mr, Nr = 65536 // scale, 768
        xr_, rr_, ghr, gnr = (torch.randn(Mr, Nr, device=dev).to(torch.bfloat16) for _ in range(4))
        wr_ = torch.randn(Nr, device=dev).to(torch.bfloat16)
        hr_, _ = _ak.fused_res_rmsnorm_fwd(xr_, rr_, wr_)
        E = Mr * Nr
        timeit(lambda: _ak.fused_res_rmsnorm_fwd(xr_, rr_, wr_), 8 * E, "fused_res_rmsnorm_fwd_bf16_65536x768", steps,
               graph=True)
        timeit(lambda: _ak.fused_res_rmsnorm_bwd(hr_, wr_, ghr, gnr), 8 * E, "fused_res_rmsnorm_bwd_bf16_65536x768",
               steps, graph=True)
        del xr_, rr_, ghr, gnr, hr_
        torch.cuda.empty_cache()

    if want("silu_gate"):
        # SiLU gate multiply bf16 [65536, 2048] (the hybrid's SwiGLU hidden width; 268 MB per tensor):
        # fwd reads gate, up, writes y; bwd reads gate, up, dy, writes d gate, d up.
        Ms, Hs = 65536 // scale, 2048
        gs_, us_, dys = (torch.randn(Ms, Hs, device=dev).to(torch.bfloat16) for _ in range(3))
        E = Ms * Hs
        timeit(lambda: _ak.silu_gate_mul_fwd(gs_, us_), 6 * E, "silu_gate_mul_fwd_bf16_65536x2048", steps, graph=True)
        timeit(lambda: _ak.silu_gate_mul_bwd(gs_, us_, dys), 10 * E, "silu_gate_mul_bwd_bf16_65536x2048", steps,
               graph=True)
        del gs_, us_, dys
        torch.cuda.empty_cache()

    if want("rope"):
        # RoPE bf16 q (64, 12, 2048, 64) read from a packed (64, 2048, 1536) QKV projection, written
        # head-major (201 MB read + 201 MB written); bwd on a dense gradient of the same shape.
        Bq, T, H, KH, hd = 64 // scale, 2048, 12, 4, 64
        qkv = torch.randn(Bq, T, (H + 2 * KH) * hd, device=dev).to(torch.bfloat16)
        qv = qkv[..., :H * hd].view(Bq, T, H, hd).transpose(1, 2)
        inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd))
        ang = torch.outer(torch.arange(T, device=dev, dtype=torch.float32), inv)
        cq, sq = ang.cos(), ang.sin()
        dyq = torch.randn(Bq, H, T, hd, device=dev).to(torch.bfloat16)
        E = Bq * H * T * hd
        timeit(lambda: _ak.rope_fwd(qv, cq, sq), 4 * E, "rope_fwd_bf16_q_64x12x2048x64_from_packed_qkv", steps,
               graph=True)
        timeit(lambda: _ak.rope_bwd(dyq, cq, sq), 4 * E, "rope_bwd_bf16_64x12x2048x64", steps, graph=True)
        del qkv, qv, dyq
        torch.cuda.empty_cache()

    if want("conv1d"):
        # Depthwise causal conv1d + SiLU bf16 (16, 1536, 2048), K=4 (the Mamba block's
        # conv at the hybrid model's d_inner): 100 MB per tensor, x + y > L2.
        Bsz, Dc, T = max(1, 16 // scale), 1536, 2048
        xc = torch.randn(Bsz, Dc, T, device=dev).to(torch.bfloat16)
        dyc = torch.randn(Bsz, Dc, T, device=dev).to(torch.bfloat16)
        wc, bc = torch.randn(Dc, 4, device=dev), torch.randn(Dc, device=dev)
        E = Bsz * Dc * T
        timeit(lambda: _ak.causal_conv1d_fwd(xc, wc, bc, True), 4 * E, "conv1d_silu_fwd_bf16_16x1536x2048", steps,
               graph=True)
        timeit(lambda: _ak.causal_conv1d_bwd(xc, wc, bc, dyc, True), 6 * E, "conv1d_silu_bwd_bf16_16x1536x2048",
               steps, graph=True)
        del xc, dyc
        torch.cuda.empty_cache()
    if scale != 1:
        res["_ops_scale"] = scale
    return res


def time_sharded_ops(dev, world, rank, steps, warmup, hbm_peak, bf16_peak):
    """Strong scaling of the per-op BASELINE configs (the split of kernels/sharded.py): each
    config's rows are split over the `world` ranks and every rank runs its block; the collectives
    the split needs (linear + CE: valid count, loss and dW; scan: dA, dD, ddelta_bias) run inside
    the timed region on the launching stream.  t_N = max over ranks of the CUDA-event time per
    step.  t_1 = the whole config on one GPU, measured in the same run on every rank's own GPU at
    once (no data is shared, so the ranks do not disturb each other) and max-reduced.  Efficiency
    = t_1 / (N * t_N).  Each repetition is preceded by a 256 MB write that flushes L2 (its own
    time, measured alone, is subtracted), so a block that fits in L2 is not read from it."""
    from kernels import _ak, sharded
    st = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def timed(fn, reps):
        for _ in range(warmup):
            flush.zero_()
            fn()
        torch.cuda.synchronize(dev)
        barrier(world)
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(st)
        for _ in range(reps):
            flush.zero_()
        b.record(st)
        for _ in range(reps):
            flush.zero_()
            fn()
        c.record(st)
        torch.cuda.synchronize(dev)
        return max(b.elapsed_time(c) - a.elapsed_time(b), 1e-6) / reps  # (flush + op) - flush

    res = {}

    def report(name, t1, tn, amount, unit, peak, **extra):
        t1 = max_over_ranks(t1, world, dev)
        tn = max_over_ranks(tn, world, dev)
        agg = amount / (tn / 1e3) / (1e9 if unit == "GB/s" else 1e12)
        # frac: aggregate over the sum of the ranks' peaks
        res[name] = {"ms_1gpu": round(t1, 4), "ms_sharded": round(tn, 4), unit: round(agg, 1),
                     "frac_per_gpu": round(agg / (world * peak), 3), "efficiency": round(t1 / (world * tn), 3),
                     **extra}

    def both(full_fn, local_fn, reps):
        # the collectives in local_fn need every rank; full_fn runs on every rank's own GPU
        return timed(full_fn, reps), timed(local_fn, reps)

    # RMSNorm fp32 [8192, 768] fwd + bwd (config 0); the global dW is all-reduced (768 floats)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(8192, 768, generator=gen).to(dev)
    w = (1 + 0.02 * torch.randn(768, generator=gen)).to(dev)
    dy = torch.randn(8192, 768, generator=gen).to(dev)
    xl, dyl = sharded.local_rows(x), sharded.local_rows(dy)
    # dW left as this rank's partial sum (in data-parallel training the gradient all-reduce sums
    # it); the time with its own 768-float all-reduce is reported beside it
    t1, tn = both(lambda: (_ak.rmsnorm_fwd(x, w, 1e-6), _ak.rmsnorm_bwd(x, w, dy, 1e-6)),
                  lambda: (_ak.rmsnorm_fwd(xl, w, 1e-6),
                           sharded.rmsnorm_bwd_sharded(xl, w, dyl, 1e-6, global_dw=False)), steps * 2)
    tg = timed(lambda: (_ak.rmsnorm_fwd(xl, w, 1e-6), sharded.rmsnorm_bwd_sharded(xl, w, dyl, 1e-6)), steps * 2)
    E = 8192 * 768
    report("rmsnorm_fp32_8192x768_fwd_bwd", t1, tn, 5 * E * 4 + 3 * 768 * 4, "GB/s", hbm_peak,
           ms_sharded_with_dw_allreduce=round(max_over_ranks(tg, world, dev), 4))
    del x, dy, xl, dyl

    # Softmax causal bf16 [196608, 2048] fwd + bwd (config 3)
    rows, cols = 96 * 2048, 2048
    s = (torch.randn(rows, cols, device=dev) / 8).to(torch.bfloat16)
    r = torch.arange(rows, device=dev) % cols
    s.masked_fill_(torch.arange(cols, device=dev)[None, :] > r[:, None], float("-inf"))
    dys = torch.randn(rows, cols, device=dev).to(torch.bfloat16)
    sl, dysl = sharded.local_rows(s), sharded.local_rows(dys)
    t1, tn = both(lambda: _ak.softmax_bwd(_ak.softmax_fwd(s), dys),
                  lambda: _ak.softmax_bwd(_ak.softmax_fwd(sl), dysl), steps)
    report("softmax_bf16_196608x2048_fwd_bwd", t1, tn, 5 * rows * cols * 2, "GB/s", hbm_peak)
    del s, dys, sl, dysl, r
    torch.cuda.empty_cache()

    # Mamba selective scan (config 1): batch rows 8 / N per rank; dA, dD, ddelta_bias all-reduced
    cfg = dict(HEADLINE)
    host = make_sscan_inputs(cfg, dev, seed=1234)
    d = {k: v.to(dev) for k, v in host.items()}
    dl = {k: (sharded.local_rows(v) if v.dim() == 3 else v) for k, v in d.items()}

    def scan(t, collect):
        out, last, states = _ak.selective_scan_fwd(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                                   t["delta_bias"], True)
        gr = _ak.selective_scan_bwd(t["dout"], t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                    t["delta_bias"], True, states)
        if collect:
            sharded.selective_scan_bwd_sharded(gr)

    t1, tn = both(lambda: scan(d, False), lambda: scan(dl, True), steps)
    fb, bb = sscan_bytes(cfg["batch"], cfg["dim"], cfg["L"], cfg["N"], cfg["groups"])
    report("selective_scan_bf16_B8_D1536_L2048_N16_fwd_bwd", t1, tn, fb + bb, "GB/s", hbm_peak)
    del d, dl, host
    torch.cuda.empty_cache()

    # Linear + CE bf16 (config 2): tokens 32768 / N per rank, W replicated; valid count, loss and
    # dW (bf16, 77 MB) all-reduced
    Nt, Dh, Vv = 32768, 768, 50304
    gen = torch.Generator().manual_seed(0)
    H = torch.randn(Nt, Dh, generator=gen).to(torch.bfloat16).to(dev)
    W = (torch.randn(Vv, Dh, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
    lab = torch.randint(0, 50257, (Nt,), generator=gen)
    lab[torch.randperm(Nt, generator=gen)[: Nt // 20]] = -100
    lab = lab.to(dev)
    Hl, labl = sharded.local_rows(H), sharded.local_rows(lab)
    reps = max(3, steps // 4)
    t1, tn = both(lambda: _ak.linear_ce_fwdbwd(H, W, lab, -100),
                  lambda: sharded.linear_ce_sharded(Hl, W, labl, -100), reps)
    report("linear_ce_bf16_32768x768x50304_fwd_bwd", t1, tn, 3 * 2 * Nt * Dh * Vv, "TFLOP/s", bf16_peak)
    del H, W, lab, Hl, labl, flush
    torch.cuda.empty_cache()
    return {"n_gpus": world, "scaling": "strong (fixed total work split over the ranks)",
            "l2": "256 MB write before each repetition, its time subtracted", **res}


def profile_train_step(dev, micro_batch=16, seq=1024):
    """One 124M training step (the CUDA-graph step the bench times) bracketed by
    cudaProfilerStart / Stop after the eager warm-up, capture and one replay."""
    from halo_training.hybrid_lm import HybridConfig
    from halo_training.train_step import HybridTrainer, synthetic_batch
    torch.cuda.set_device(dev)
    cfg = HybridConfig()
    tr = HybridTrainer(cfg, device=dev, use_kernels=True, seed=0, cuda_graph=True)
    idx, tgt = synthetic_batch(micro_batch, seq, cfg.vocab_size, seed=1000, device=dev)
    for _ in range(tr.graph_warmup + 2):
        tr.step(idx, tgt)
    torch.cuda.synchronize(dev)
    torch.cuda.cudart().cudaProfilerStart()
    tr.step(idx, tgt)
    torch.cuda.synchronize(dev)
    torch.cuda.cudart().cudaProfilerStop()


def time_train(dev, steps, warmup, world, rank, micro_batch=16, seq=1024):
    """124M hybrid training step: kernels swapped in through the
    reference-facing API, bf16 autocast, AdamW, DDP over NCCL when world > 1."""
    from halo_training.hybrid_lm import HybridConfig, count_params
    from halo_training.train_step import HybridTrainer, synthetic_batch
    cfg = HybridConfig()
    # the whole step (forward, backward with DDP's all-reduce, AdamW) replays as one CUDA graph
    tr = HybridTrainer(cfg, device=dev, use_kernels=True, ddp=world > 1, seed=0, cuda_graph=True)
    idx, tgt = synthetic_batch(micro_batch, seq, cfg.vocab_size, seed=1000 + rank, device=dev)
    st = torch.cuda.current_stream(dev)
    for _ in range(max(warmup, tr.graph_warmup + 2)):  # eager warm-up, capture, one replay
        tr.step(idx, tgt)
    torch.cuda.synchronize(dev)
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(steps):
        loss = tr.step(idx, tgt)
    b.record(st)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(a.elapsed_time(b) / steps, world, dev)
    out = {"tok_s": round(world * micro_batch * seq / (ms / 1e3), 1), "ms_per_step": round(ms, 3),
           "params": count_params(tr.raw), "micro_batch_per_gpu": micro_batch, "seq_len": seq,
           "loss_last": round(float(loss.item()), 4), "steps": steps,
           "model": "hybrid 12L d768 (6 Mamba N16 + 6 GQA 12q/4kv), SwiGLU 2048, tied 50304 vocab",
           "parallelism": f"ddp{world} (NCCL)" if world > 1 else "single GPU",
           "cuda_graph": "whole step (forward, backward, all-reduce, AdamW) captured once, replayed per step"}
    del tr
    torch.cuda.empty_cache()
    return out


def run_ours(args, world, rank, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm_peak, tf_peak, peak_kind = peaks()
    if args.only_ops:
        if rank == 0:
            emit({"ops": time_other_ops(dev, args.steps, args.warmup, hbm_peak, tf_peak,
                                        which=set(args.ops.split(",")) if args.ops else None,
                                        ce_rows=args.ce_rows, scale=args.ops_scale)})
        return
    cfg = dict(HEADLINE)
    if args.batch:
        cfg["batch"] = args.batch  # profiling / small-case runs only
    total_ms, fwd_ms, bwd_ms, clocks, host = time_sscan(cfg, dev, args.steps, args.warmup, world)
    total_ms = max_over_ranks(total_ms, world, dev)
    fwd_b, bwd_b = sscan_bytes(cfg["batch"], cfg["dim"], cfg["L"], cfg["N"], cfg["groups"])
    ms_per_step = total_ms / args.steps
    value = world * (fwd_b + bwd_b) / (ms_per_step / 1e3) / 1e9
    bwd_avg = statistics.mean(bwd_ms)
    fwd_avg = statistics.mean(fwd_ms)
    achieved = bwd_b / (bwd_avg / 1e3) / 1e9
    traffic = NCU_TRAFFIC_BYTES.get("sscan_bwd")
    inst = NCU_WARP_INST["sscan_bwd"] * cfg["batch"] / 8
    sm_mhz = clocks.get("sm_mhz") or 1965.0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    issue_peak = sms * 4 * sm_mhz * 1e6 / 1e9  # G warp-instructions / s
    issue_achieved = inst / (bwd_avg / 1e3) / 1e9
    if args.no_e2e:
        e2e_ms, h2d, d2h, e2e_value, copy_ms = float("nan"), 0, 0, None, float("nan")
    else:
        e2e_ms, h2d, d2h, copy_ms = time_sscan_e2e(cfg, dev, max(2, args.steps // 2), 2, host)
        e2e_ms = max_over_ranks(e2e_ms, world, dev)
        copy_ms = max_over_ranks(copy_ms, world, dev)
        e2e_value = round(world * (fwd_b + bwd_b) / (e2e_ms / 1e3) / 1e9, 2)
    comparator = None
    if rank == 0 and world == 1 and not args.no_comparator:
        comparator = time_comparator(dev, host, args.steps, args.warmup, fwd_avg, bwd_avg)
    ops = time_other_ops(dev, args.steps, args.warmup, hbm_peak, tf_peak) if (rank == 0 and not args.no_ops) else None
    train = None if args.no_train else time_train(dev, args.train_steps, 3, world, rank)
    sharded = None
    if not args.no_sharded:
        sharded = time_sharded_ops(dev, world, rank, args.steps, args.warmup, hbm_peak, tf_peak)
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config 1 distributions)",
        "config": {"workload": "mamba selective_scan fwd+bwd B=8 D=1536 L=2048 N=16 bf16, fp32 state, "
                               "softplus(delta+bias), SiLU(z), last_state",
                   "per_rank_batch": cfg["batch"], "global_batch": cfg["batch"] * world,
                   "parallelism": f"rows sharded over {world} GPU(s), no data-path collective",
                   "l2": "no flush: per-step working set 558 MB > 126 MB L2",
                   "fwd_ms": round(fwd_avg, 4), "bwd_ms": round(bwd_avg, 4),
                   "fwd_GBps": round(fwd_b / (fwd_avg / 1e3) / 1e9, 1),
                   "sfu_exp2_per_pass": cfg["batch"] * cfg["dim"] * cfg["L"] * cfg["N"]},
        "roofline": {"kernel": "selective_scan_bwd (C-ABI call)", "bound": "issue",
                     "achieved": round(issue_achieved, 1), "peak": round(issue_peak, 1),
                     "unit": "G warp-instructions/s", "frac": round(issue_achieved / issue_peak, 4),
                     "warp_instructions_per_launch": int(inst),
                     "issue_peak_def": f"{sms} SMs x 4 schedulers x 1 warp-instruction/clk at the sampled "
                                       f"median SM clock {sm_mhz:.0f} MHz; instructions from ncu "
                                       "smsp__inst_executed.sum",
                     "hbm": {"achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                             "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind},
                     "traffic": traffic, "algorithmic_bytes_per_launch": bwd_b},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "copy_bound": {"h2d_only_ms": round(copy_ms, 3),
                               "h2d_GBps": round(h2d / (copy_ms / 1e3) / 1e9, 1) if copy_ms == copy_ms else None,
                               "frac": round(copy_ms / e2e_ms, 3) if e2e_ms == e2e_ms else None,
                               "def": "the step's H2D copies alone (pinned, same slicing, copy stream, "
                                      "CUDA events); frac = h2d_only_ms / ms_per_step"},
                "api": "kernels.mamba_scan.selective_scan_fn + autograd backward, pinned host inputs, "
                       "H2D of batch slice i+1 overlapped with fwd+bwd of slice i (8 slices of one batch row)"},
        # per timed step: sscan_fwd_kernel; sscan_bwd_kernel, sscan_bwd_reduce, f32_to2 (dB and dC)
        "gpu_launches": 4 * args.steps,
        "clocks": clocks,
    }
    if comparator is not None:
        line["comparator"] = comparator
    if ops is not None:
        line["ops"] = ops
    if train is not None:
        line["train"] = train
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_sscan_sample()
        if not args.no_ops:
            line["cpu_baseline"]["ops"] = cpu_ops_sample()["ops"]
    if sharded is not None:
        line["sharded_ops"] = sharded
    # last key, so a tail of the output still carries every op's roofline fraction
    summary = {}
    if ops is not None:
        for k, v in ops.items():
            if isinstance(v, dict):
                f = v.get("frac", v.get("frac_bf16"))
                if f is not None:
                    summary[k] = f
                if isinstance(v.get("rotating_buffers"), dict):
                    summary[k + "_rotating"] = v["rotating_buffers"]["frac"]
                if k.startswith("linear_ce_gemms_vs_cublas"):
                    for name, c in v.items():
                        summary[f"tc_gemm_{name}_vs_cublas"] = c["ratio_vs_cublas"]
    if copy_ms == copy_ms and e2e_ms == e2e_ms:
        summary["e2e_frac_of_h2d_copy_bound"] = round(copy_ms / e2e_ms, 3)
    if train is not None:
        summary["train_tok_s"] = train["tok_s"]
    if comparator is not None and "speedup_total" in comparator:
        summary["scan_speedup_vs_reference_cuda"] = comparator["speedup_total"]
        summary["scan_bwd_speedup_vs_reference_cuda"] = comparator["speedup_bwd"]
    if sharded is not None:
        for k, v in sharded.items():
            if isinstance(v, dict) and "efficiency" in v:
                summary[f"sharded_eff_{k}"] = v["efficiency"]
    line["ops_summary"] = summary
    emit(line)


def run_reference(args, world, rank):
    """The reference's CPU path (the oracle port of selective_scan_ref + autograd), timed on
    the host cores on a bounded sample of the headline workload; rank 0 only."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        cpu_sscan_sample(dim_sample=8, L=512)
    samples = [cpu_sscan_sample() for _ in range(args.steps)]
    v = statistics.median(s["value"] for s in samples)
    cb = dict(samples[0])
    cb["value"] = v
    fwd_b, bwd_b = sscan_bytes(1, 48, 2048, 16, 1)
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round((fwd_b + bwd_b) / (v * 1e9) * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config 1 distributions)",
            "config": {"workload": "mamba selective_scan fwd+bwd, bounded CPU sample of B=8 D=1536 L=2048 N=16"},
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


# The JSON result goes to the original stdout; everything else the process writes
# to fd 1 (library banners such as NCCL's version line) is sent to stderr.
_JSON_OUT = None


def emit(obj) -> None:
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-op sweep")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-train", action="store_true", help="skip the 124M hybrid training step")
    ap.add_argument("--train-steps", type=int, default=10)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sharded", action="store_true", help="skip the strong-scaled per-op block")
    ap.add_argument("--no-comparator", action="store_true", help="skip timing the reference's own CUDA scan")
    ap.add_argument("--only-ops", action="store_true", help="print only the per-op sweep (quick runs)")
    ap.add_argument("--ops", default="", help="with --only-ops: comma list of rmsnorm,softmax,linear_ce,scan1,ce_rows,fused_res,silu_gate,rope,conv1d")
    ap.add_argument("--ce-rows", type=int, default=32768, help="with --only-ops: rows of the linear+CE case")
    ap.add_argument("--ops-scale", type=int, default=1,
                    help="with --only-ops: divide the leading dimension of the softmax, fused_res, silu_gate, rope "
                         "and conv1d cases by this (small cases for ncu captures; names keep the full-size label)")
    ap.add_argument("--batch", type=int, default=0, help="override the headline batch (small-case profiling)")
    ap.add_argument("--profile-train", action="store_true",
                    help="profiling mode: warm the 124M training step up, then run exactly one step between "
                         "cudaProfilerStart / Stop (for ncu --profile-from-start off); prints no JSON")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = setup_dist()
    if args.profile_train:
        profile_train_step(torch.device("cuda", local))
        return
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
