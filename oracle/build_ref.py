"""Builds the reference's own CUDA extension into oracle/_ref (two modules).

TEST INFRASTRUCTURE ONLY. Both compile UNMODIFIED reference sources, where they lie under the
reference checkout, for sm_100a with the reference's default nvcc flags otherwise (it ships
none; reference setup.py:64-79):

* `ref_raster`: csrc/forward/rasterize.cu and csrc/backward/rasterize_backward.cu (the
  binning, sort and blend kernels, which need no third-party header) with ref_raster_bind.cpp.
* `ref_full` ("ref+shim"): the whole extension as the reference's setup.py lists it --
  csrc/bindings.cpp and all six .cu files, so the module exposes the reference's six ops
  (`project`, `SH`, `rasterize`, `backwards_rasterization`, `backwards_SH`,
  `backwards_projection`) under their own names. projection.cu, SH.cu,
  projection_backward.cu and delight_backward.cu include GLM, which the reference does not
  vendor or pin and which is absent from this image; oracle/glm_shim supplies the API subset
  they use, restated from GLM's documented semantics. Results of these four files are
  therefore "ref+shim": the reference's expressions over that restatement.

Usage: python oracle/build_ref.py [--reference /path/to/reference]
The modules are importable afterwards as `ref_raster` / `ref_full` with oracle/_ref on
sys.path (the built .so files travel with the repository snapshot; the reference checkout
itself is needed only to build them).
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


FULL_SOURCES = ("bindings.cpp", "forward/projection.cu", "forward/rasterize.cu", "forward/SH.cu",
                "backward/rasterize_backward.cu", "backward/projection_backward.cu",
                "backward/delight_backward.cu")


def _load(name: str, sources: list[Path], includes: list[Path], verbose: bool) -> Path | None:
    from torch.utils import cpp_extension

    out = OUT / name
    out.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name=name,
        sources=[str(p) for p in sources],
        extra_include_paths=[str(p) for p in includes],
        extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=str(out),
        verbose=verbose,
        with_cuda=True,
    )
    libs = sorted(out.glob(f"{name}*.so"))
    return libs[0] if libs else None


def build(reference: Path = DEFAULT_REFERENCE, verbose: bool = False) -> list[Path]:
    csrc = reference / "csrc"
    raster = [csrc / "forward" / "rasterize.cu", csrc / "backward" / "rasterize_backward.cu"]
    full = [csrc / f for f in FULL_SOURCES]
    if not all(p.exists() for p in full):
        return []
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    inc = [csrc, csrc / "forward", csrc / "backward"]
    built = [
        _load("ref_raster", [HERE / "ref_raster_bind.cpp", *raster], inc, verbose),
        _load("ref_full", full, [*inc, HERE / "glm_shim"], verbose),
    ]
    return [p for p in built if p is not None]


def module_dirs() -> list[str]:
    """Directories to put on sys.path to import ref_raster / ref_full."""
    return [str(OUT / "ref_raster"), str(OUT / "ref_full")]


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    paths = build(args.reference, args.verbose)
    print("\n".join(map(str, paths)) if paths else "reference sources not found; nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
