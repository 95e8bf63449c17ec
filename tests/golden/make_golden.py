"""Generates the golden vectors tests/golden/ref_raster_*.npz and ref_gaussian_*.npz on a CUDA
machine, from the REFERENCE's own kernels built by oracle/build_ref.py.

* ref_raster_*: inputs (mean2d, cov2d, depths, colors, opacity) come from the CPU oracle's
  projection and SH of seeded scenes; the outputs come from the reference's binning / blend
  kernels (csrc/forward/rasterize.cu, csrc/backward/rasterize_backward.cu, built unmodified,
  module ref_raster).
* ref_gaussian_*: the per-Gaussian stages -- `project`, `SH`, `backwards_SH`,
  `backwards_projection` (csrc/forward/projection.cu, csrc/forward/SH.cu,
  csrc/backward/delight_backward.cu, csrc/backward/projection_backward.cu) -- of the
  reference's whole extension built against the GLM stand-in oracle/glm_shim (module ref_full,
  "ref+shim"), on seeded Gaussians, cameras and upstream gradients stored in the file.

The files pin the oracle (tests/test_oracle_kat.py) and the CUDA path (tests/test_gpu_parity.py,
tests/test_gpu_ref_shim.py) to the reference's behaviour.

Usage (GPU box): python tests/golden/make_golden.py [--out DIR] [--only raster|gaussian]
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


def gaussian_cases():
    """(name, scene, view): 1,024 Gaussians each (small files), plus hand-made edge rows."""
    sc0 = scenes.config0(0)
    yield "config0", sub_scene(sc0, 0, 1024, edge_rows=True), sc0.views[0]
    sc1 = scenes.config1(0)
    yield "config1_1080", sub_scene(sc1, 5000, 1024), sc1.views[1]
    behind = scenes.config0(2)
    yield "partly_behind_camera", sub_scene(behind, 0, 1024), scenes.pinhole(
        (0.0, 0.0, 0.5), 96, 64, 64.0)


def sub_scene(sc, start, n, edge_rows=False):
    p = [x[start:start + n].clone() for x in sc.params()]
    if edge_rows:
        # a zero quaternion (normalised to the identity), an unnormalised one, a quaternion with
        # a negative real part, extreme log-scales, a Gaussian just in front of the near plane
        # and one just behind it (camera at z = 4 looking down -z: depth = 4 - z)
        mu, q, s = p[0], p[1], p[2]
        q[0] = 0.0
        q[1] = torch.tensor([3.0, -1.0, 0.5, 2.0])
        q[2] = torch.tensor([-0.9, 0.1, 0.3, -0.2])
        s[3] = torch.tensor([-12.0, -12.0, -12.0])
        s[4] = torch.tensor([1.5, -9.0, 0.5])
        mu[5] = torch.tensor([0.01, -0.02, 4.0 - 0.2001])
        mu[6] = torch.tensor([0.01, -0.02, 4.0 - 0.2])
    return scenes.Scene(sc.name, *p)


def make_gaussian(name, sc, view, ref, out_dir: Path, seed: int):
    dev = torch.device("cuda")
    mu, q, s, _, A, kj = [x.to(dev).contiguous() for x in sc.params()]
    R, t = view.R.to(dev).contiguous(), view.T.to(dev).contiguous()
    cam = (-(R.T @ t)).contiguous()
    N = sc.N
    mean2d, cov2d, depths = ref.project(N, mu, q, s, R, t, view.fx, view.fy, view.cx, view.cy)
    colors = ref.SH(N, cam, mu, A, kj)
    g = torch.Generator("cpu").manual_seed(seed)
    g_colors = torch.randn(N, 3, generator=g).to(dev)
    g_mean2d = torch.randn(N, 2, generator=g).to(dev)
    g_cov2d = (0.1 * torch.randn(N, 3, generator=g)).to(dev)
    gA, gkj, gmu_sh = ref.backwards_SH(g_colors, mu, A, kj, cam)
    gmu, gq, gs = ref.backwards_projection(g_mean2d, g_cov2d, mu, q, s, R, t, view.fx, view.fy,
                                           view.cx, view.cy)
    torch.cuda.synchronize()
    cpu = lambda x: x.detach().cpu().numpy()  # noqa: E731
    path = out_dir / f"ref_gaussian_{name}.npz"
    np.savez_compressed(
        path, mu=cpu(mu), q=cpu(q), s=cpu(s), A=cpu(A), k_j=cpu(kj), R=cpu(R), t=cpu(t),
        cam=cpu(cam), intr=np.array([view.fx, view.fy, view.cx, view.cy], np.float32),
        mean2d=cpu(mean2d), cov2d=cpu(cov2d), depths=cpu(depths), colors=cpu(colors),
        g_colors=cpu(g_colors), g_mean2d=cpu(g_mean2d), g_cov2d=cpu(g_cov2d), g_A=cpu(gA),
        g_k_j=cpu(gkj), g_mu_sh=cpu(gmu_sh), g_mu=cpu(gmu), g_q=cpu(gq), g_s=cpu(gs))
    print(f"{path.name}: N={N} culled={int((depths == 0).sum())}", flush=True)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--out", type=Path, default=Path(__file__).resolve().parent)
    ap.add_argument("--only", choices=("raster", "gaussian"), default=None)
    args = ap.parse_args()
    args.out.mkdir(parents=True, exist_ok=True)
    if args.only in (None, "raster"):
        import ref_raster as ref  # built by oracle/build_ref.py

        for k, (name, sc, view) in enumerate(cases()):
            make(name, sc, view, ref, args.out, seed=100 + k)
    if args.only in (None, "gaussian"):
        import ref_full  # built by oracle/build_ref.py (ref+shim)

        for k, (name, sc, view) in enumerate(gaussian_cases()):
            make_gaussian(name, sc, view, ref_full, args.out, seed=200 + k)
    return 0


if __name__ == "__main__":
    sys.exit(main())
