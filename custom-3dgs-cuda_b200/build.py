"""Builds the sm_100a shared library libgs3d_b200.so from csrc/*.cu with nvcc.

Objects go to _build/ next to this file; the library lands inside the
custom_rasterizer_cuda package so the Python boundary loads it from the source tree.
Compilation is incremental (by modification time, including headers) and parallel.

Usage: python build.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "custom_rasterizer_cuda" / "libgs3d_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libgs3d_b200")
    return found


def _newest_header() -> float:
    heads = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in heads), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool, extra: list[str]) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(src),
           "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout, res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles every csrc/*.cu for sm_100a and links libgs3d_b200.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    head_time = _newest_header()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        stale = (force or ptxas_info or not obj.exists()
                 or obj.stat().st_mtime < max(src.stat().st_mtime, head_time))
        if stale:
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(workers) as pool:
            futs = [pool.submit(_compile, s, o, verbose or ptxas_info, extra) for s, o in jobs]
            for f in futs:
                f.result()
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-rdc=true", "-shared", "-Xcompiler", "-fPIC",
               *map(str, objs), "-o", str(tmp), "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true",
                    help="recompile with -Xptxas -v to print registers, spills and shared memory")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
