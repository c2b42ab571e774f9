"""Build the reference's own mamba selective-scan CUDA extension (`selective_scan_cuda`) for
sm_100a into `oracle/_ref/mamba/` — TEST / BENCH INFRASTRUCTURE ONLY.

It is the GPU comparator for the headline selective scan: the vendored mamba_ssm 2.3.0 kernels
(external/mamba/csrc/selective_scan/*, cub block scans, SIMT) that the reference would run on a
CUDA GPU, compiled from their sources where they lie in the reference checkout with the compile
flags of external/mamba/setup.py:228-244 and the architecture set to sm_100a.  Nothing here is
part of the product path; tests/test_gpu_mamba_comparator.py checks parity with it and asserts that
our scan is faster than it at the headline configuration, and bench.py times it beside our scan on the
same inputs (its `comparator` entry) when the module has been built.

    python oracle/build_mamba_ref.py [--reference PATH] [--jobs N]

The build needs the reference checkout (not the GPU box); the built .so travels to the box.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "mamba"

SOURCES = [
    "selective_scan.cpp",
    "selective_scan_fwd_fp32.cu", "selective_scan_fwd_fp16.cu", "selective_scan_fwd_bf16.cu",
    "selective_scan_bwd_fp32_real.cu", "selective_scan_bwd_fp32_complex.cu",
    "selective_scan_bwd_fp16_real.cu", "selective_scan_bwd_fp16_complex.cu",
    "selective_scan_bwd_bf16_real.cu", "selective_scan_bwd_bf16_complex.cu",
]

NVCC_FLAGS = [
    "-O3", "-std=c++17",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
    "--expt-relaxed-constexpr", "--expt-extended-lambda", "--use_fast_math", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a", "--threads", "4",
]


def built_module_path() -> Path:
    return OUT / "selective_scan_cuda.so"


def load_built():
    """Import the built comparator (None when it has not been built)."""
    p = built_module_path()
    if not p.exists():
        return None
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the extension links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader("selective_scan_cuda", str(p))
    spec = importlib.util.spec_from_file_location("selective_scan_cuda", str(p), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def default_reference() -> Path:
    """$AK_REFERENCE, else a `reference` checkout beside this repository."""
    return Path(os.environ.get("AK_REFERENCE", str(Path(__file__).resolve().parents[2] / "reference")))


def build(reference: Path | None = None, jobs: int | None = None, verbose: bool = False) -> Path | None:
    """Compile (incrementally, through ninja) the comparator into oracle/_ref/mamba/; returns the
    module path, or None when the reference sources are not present."""
    src = Path(reference or default_reference()) / "external" / "mamba" / "csrc" / "selective_scan"
    if not src.is_dir():
        if verbose:
            print(f"reference sources not found at {src}; nothing built", file=sys.stderr)
        return None
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(jobs or os.cpu_count() or 4))
    from torch.utils.cpp_extension import load
    load(name="selective_scan_cuda", sources=[str(src / s) for s in SOURCES],
         extra_cflags=["-O3", "-std=c++17"], extra_cuda_cflags=NVCC_FLAGS, extra_include_paths=[str(src)],
         build_directory=str(OUT), verbose=verbose)
    return built_module_path()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(default_reference()))
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    args = ap.parse_args()
    out = build(Path(args.reference), args.jobs, verbose=True)
    if out is not None:
        print("built", out)


if __name__ == "__main__":
    main()
