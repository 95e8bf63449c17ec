"""Generates the golden vectors tests/golden/ref_raster_*.npz on a CUDA machine.

Inputs (mean2d, cov2d, depths, colors, opacity) come from the CPU oracle's projection and SH
of seeded scenes; the outputs come from the REFERENCE's own binning / blend kernels
(csrc/forward/rasterize.cu, csrc/backward/rasterize_backward.cu, built unmodified into
oracle/_ref by oracle/build_ref.py). The files pin the oracle (tests/test_oracle_kat.py) and
the CUDA path (tests/test_gpu_parity.py) to the reference's behaviour.

Usage (GPU box): python tests/golden/make_golden.py [--out DIR]
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT), str(ROOT / "custom-3dgs-cuda_b200"), str(ROOT / "oracle" / "_ref" / "ref_raster"),
                str(ROOT / "oracle" / "_ref" / "ref_full")]

from gs3d_b200 import scenes  # noqa: E402
from oracle import oracle as O  # noqa: E402


def cases():
    """(name, scene, view) with small sizes: config 0, a reduced clustered scene, odd image
    sizes, a scene partly behind the camera, and one splat per tile row edge."""
    sc0 = scenes.config0(0)
    yield "config0", sc0, sc0.views[0]
    sc2 = scenes.config2(0, n=20_000)
    yield "clustered20k_256x144", sc2, scenes.pinhole((0.0, 0.0, 8.0), 256, 144, 200.0)
    sc1 = scenes.config1(1)
    sub = scenes.Scene("config1_sub", *(p[:12_000] for p in sc1.params()))
    yield "uniform12k_100x70", sub, scenes.pinhole((0.0, 0.0, 6.0), 100, 70, 80.0)
    behind = scenes.config0(2)
    yield "config0_partly_behind_camera", behind, scenes.pinhole((0.0, 0.0, 0.5), 96, 64, 64.0)


def make(name, sc, view, ref, out_dir: Path, seed: int):
    R, t = view.R.numpy(), view.T.numpy()
    mean2d, cov2d, depths = O.project(sc.mu.numpy(), sc.q.numpy(), sc.s.numpy(), R, t, view.fx,
                                      view.fy, view.cx, view.cy)
    colors = O.sh(O.camera_position(R, t), sc.mu.numpy(), sc.A.numpy(), sc.k_j.numpy())
    alpha = torch.sigmoid(sc.alpha).numpy().reshape(-1, 1).astype(np.float32)
    H, W = view.height, view.width
    dev = torch.device("cuda")
    tens = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in
            dict(mean2d=mean2d, cov2d=cov2d, depths=depths, colors=colors, alpha=alpha).items()}
    img, ids, ranges, final_T, n_contrib = ref.rasterize(
        sc.N, tens["depths"], tens["mean2d"], tens["cov2d"], tens["colors"], tens["alpha"], H, W)
    g = torch.Generator("cpu").manual_seed(seed)
    grad_img = torch.rand(H, W, 3, generator=g).to(dev)
    gm, gc, gcol, ga = ref.backwards_rasterization(
        grad_img, tens["mean2d"], tens["cov2d"], tens["colors"], tens["alpha"], ids, ranges,
        final_T, n_contrib, sc.N, H, W)
    torch.cuda.synchronize()
    cpu = lambda x: x.detach().cpu().numpy()  # noqa: E731
    path = out_dir / f"ref_raster_{name}.npz"
    np.savez_compressed(
        path, H=H, W=W, mean2d=mean2d, cov2d=cov2d, depths=depths, colors=colors,
        alpha=alpha.reshape(-1), img=cpu(img), sorted_ids=cpu(ids), tile_ranges=cpu(ranges),
        final_T=cpu(final_T), n_contrib=cpu(n_contrib), grad_img=cpu(grad_img),
        g_mean2d=cpu(gm), g_cov2d=cpu(gc), g_colors=cpu(gcol), g_alpha=cpu(ga))
    print(f"{path.name}: N={sc.N} M={ids.numel()} {W}x{H}", flush=True)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--out", type=Path, default=Path(__file__).resolve().parent)
    args = ap.parse_args()
    import ref_raster as ref  # built by oracle/build_ref.py

    args.out.mkdir(parents=True, exist_ok=True)
    for k, (name, sc, view) in enumerate(cases()):
        make(name, sc, view, ref, args.out, seed=100 + k)
    return 0


if __name__ == "__main__":
    sys.exit(main())
