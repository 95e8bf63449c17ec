"""Builds the reference's GLM-free kernels into oracle/_ref/ref_raster*.so.

TEST INFRASTRUCTURE ONLY. Compiles the UNMODIFIED reference sources
csrc/forward/rasterize.cu and csrc/backward/rasterize_backward.cu, where they lie under the
reference checkout, together with ref_raster_bind.cpp, for sm_100a with the reference's
default nvcc flags otherwise (it ships none). The reference's projection.cu, SH.cu,
projection_backward.cu and delight_backward.cu include GLM, a third-party header library
that is not installed here, so they are not built.

Usage: python oracle/build_ref.py [--reference /path/to/reference]
The module is importable afterwards as `ref_raster` with oracle/_ref on sys.path.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
# a checkout of the reference next to this repository
DEFAULT_REFERENCE = HERE.parents[1] / "reference"


def build(reference: Path = DEFAULT_REFERENCE, verbose: bool = False) -> Path | None:
    csrc = reference / "csrc"
    sources = [csrc / "forward" / "rasterize.cu", csrc / "backward" / "rasterize_backward.cu"]
    if not all(p.exists() for p in sources):
        return None
    from torch.utils import cpp_extension

    OUT.mkdir(exist_ok=True)
    os.environ.setdefault("MAX_JOBS", "4")
    cpp_extension.load(
        name="ref_raster",
        sources=[str(HERE / "ref_raster_bind.cpp"), *map(str, sources)],
        extra_include_paths=[str(csrc), str(csrc / "forward"), str(csrc / "backward")],
        extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=str(OUT),
        verbose=verbose,
        with_cuda=True,
    )
    libs = sorted(OUT.glob("ref_raster*.so"))
    return libs[0] if libs else None


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    path = build(args.reference, args.verbose)
    print(path if path else "reference sources not found; nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
