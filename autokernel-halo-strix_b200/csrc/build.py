"""Build libak_b200.so (sm_100a) from the .cu sources in this directory.

    python autokernel-halo-strix_b200/csrc/build.py [--force] [--jobs N]

Each .cu file is compiled to an object under `_build/` (skipped when the object
is newer than its source and every header), then all objects are linked into
`autokernel-halo-strix_b200/libak_b200.so`, next to the Python packages that
load it.  nvcc cross-compiles, so this runs on machines without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
INCLUDE = REPO / "include"
BUILD = PKG / "_build"
LIB = PKG / "libak_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-DNDEBUG",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, force: bool, extra: list[str]) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}\n{res.stdout}")
    return obj, res.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = list(extra or [])
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(LIB),
               "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}\n{res.stdout}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", "-v", action="store_true", help="print ptxas -v resource usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.verbose else []
    lib = build(force=args.force or args.verbose, jobs=args.jobs, verbose=args.verbose, extra=extra)
    print(lib)


if __name__ == "__main__":
    main()
