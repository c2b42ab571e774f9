"""bench.py's measurement contract, checked on CPU.

* The algorithmic bytes the headline and its roofline are computed from: the survey's per-pass
  figures for the BASELINE scan config (B=8, D=1536, L=2048, N=16, bf16) are 203,272,192 bytes for
  the forward and 354,639,872 for the backward.
* The reference arm (`--impl reference`, the CPU path timed on the host cores) prints exactly one
  JSON line with the keys the driver reads, on the same metric and unit as the GPU arm.
"""
import json
import subprocess
import sys

from conftest import REPO


def test_sscan_algorithmic_bytes_at_the_baseline_config():
    sys.path.insert(0, str(REPO))
    import bench
    fwd, bwd = bench.sscan_bytes(8, 1536, 2048, 16, 1)
    assert (fwd, bwd) == (203_272_192, 354_639_872)
    # linear in the batch apart from the per-channel parameters, which every batch shares
    f1, b1 = bench.sscan_bytes(1, 1536, 2048, 16, 1)
    par = 1536 * 16 * 4 + 2 * 1536 * 4
    assert fwd - par == 8 * (f1 - par)


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=REPO, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["warmup"] >= 3 and d["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] in ("port", "reference")
    assert "workload" in d["config"]
