"""Generates tests/golden/ref_adc_*.npz: the reference's own adaptive density control
(gaussian_splatting/utils/adc.py:330-392 of kmurungi/custom-3dgs-cuda, imported from a local
checkout of the reference) run on small seeded CPU scenes.

Each case builds Gaussians and a torch Adam optimizer with the reference's own
`setup_optimizer` (gaussian_splatting/utils/optim.py:12-31), takes two optimizer steps on
seeded gradients so that the Adam moments are non-zero, fills the densification statistics
(`xyz_grad_accum`, `denom`, `max_radii2D`) with seeded values spread around the thresholds,
and calls `adaptive_density_control`. The split step draws its offsets with `t.normal(mean,
std)`; this script substitutes `mean + z * std` with recorded unit normals `z`, so that a
reimplementation can be fed the same `z`. Saved: the inputs, `z`, the counts and every output
(parameters and, per parameter group, `exp_avg` / `exp_avg_sq` / `step`).

Usage (any machine with the reference checkout): python tests/golden/make_adc_golden.py REF_DIR
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
NAMES = ("mu", "q", "s", "alpha", "A", "k_j")
GROUPS = ("mu", "q", "Scale", "Opacity", "Albedo Coefficient", "Illumination Coefficients")


def make_case(seed: int, n: int, *, reset_opacity: bool, max_screen: float | None,
              allow_densify: bool, max_gaussians: int, alpha_mean: float = 0.0):
    from gaussian_splatting.scene.gaussian import gaussian
    from gaussian_splatting.utils.optim import setup_optimizer

    g = torch.Generator().manual_seed(seed)
    gs = gaussian(n)
    gs.mu = torch.rand(n, 3, generator=g) * 4 - 2
    q = torch.randn(n, 4, generator=g)
    gs.q = q / q.norm(dim=1, keepdim=True)
    # log-scales around log(percent_dense * extent) = log(0.04) and the 0.1 * extent prune line
    gs.s = torch.randn(n, 3, generator=g) * 1.2 + math.log(0.04)
    gs.alpha = torch.randn(n, 1, generator=g) * 3.0 + alpha_mean
    gs.A = torch.randn(n, 3, generator=g) * 0.5
    gs.k_j = torch.randn(n, 15, 3, generator=g) * 0.05
    lrs = {"mu": 1.6e-4, "q": 1e-3, "s": 5e-3, "alpha": 5e-2, "A": 2.5e-3, "k_j": 2.5e-3}
    opt = setup_optimizer(gs, lrs)
    for _ in range(2):
        for p in (gs.mu, gs.q, gs.s, gs.alpha, gs.A, gs.k_j):
            p.grad = torch.randn(p.shape, generator=g) * 0.1
        opt.step()
    gs.xyz_grad_accum = (torch.rand(n, 1, generator=g) * 4e-4)
    gs.denom = torch.randint(0, 5, (n, 1), generator=g).float()
    gs.max_radii2D = torch.rand(n, generator=g) * 40.0
    return gs, opt, dict(reset_opacity=reset_opacity, max_screen=max_screen,
                         allow_densify=allow_densify, max_gaussians=max_gaussians)


def snapshot(gs, opt):
    out = {}
    for name, group in zip(NAMES, GROUPS):
        p = getattr(gs, name)
        out[name] = p.detach().numpy().copy()
        grp = next(gr for gr in opt.param_groups if gr["name"] == group)
        st = opt.state[grp["params"][0]]
        out[f"{name}_exp_avg"] = st["exp_avg"].numpy().copy()
        out[f"{name}_exp_avg_sq"] = st["exp_avg_sq"].numpy().copy()
        out[f"{name}_step"] = np.float32(float(st["step"]))
    return out


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("reference", type=Path)
    ap.add_argument("--out", type=Path, default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference))
    from gaussian_splatting.utils import adc

    extent = 4.0
    cases = {
        "densify_prune": dict(seed=1, n=600, reset_opacity=False, max_screen=20.0,
                              allow_densify=True, max_gaussians=500_000),
        "densify_reset_no_screen": dict(seed=2, n=500, reset_opacity=True, max_screen=None,
                                        allow_densify=True, max_gaussians=500_000),
        "over_cap_prune_only": dict(seed=3, n=400, reset_opacity=False, max_screen=25.0,
                                    allow_densify=True, max_gaussians=300),
        # every opacity below min_opacity: the reference keeps the 10% most opaque
        "all_pruned_keep_top": dict(seed=4, n=300, reset_opacity=True, max_screen=None,
                                    allow_densify=True, max_gaussians=500_000,
                                    alpha_mean=-40.0),
    }
    for name, kw in cases.items():
        seed, n = kw.pop("seed"), kw.pop("n")
        torch.manual_seed(seed)
        gs, opt, c = make_case(seed, n, **kw)
        c.pop("alpha_mean", None)
        before = snapshot(gs, opt)
        stats_in = dict(grad_accum=gs.xyz_grad_accum.numpy().copy(),
                        denom=gs.denom.numpy().copy(), max_radii=gs.max_radii2D.numpy().copy())
        zs = []
        real_normal = torch.normal

        def normal(mean, std, *a, **k):
            z = torch.randn(mean.shape, generator=torch.Generator().manual_seed(seed + 100))
            zs.append(z.numpy().copy())
            return mean + z * std

        adc.t.normal = normal
        try:
            gs, opt, counts = adc.adaptive_density_control(
                gs, opt, grad_threshold=0.00005, percent_dense=0.01, min_opacity=0.01,
                scene_extent=extent, max_screen_size=c["max_screen"],
                reset_opacity=c["reset_opacity"], max_gaussians=c["max_gaussians"],
                allow_densify=c["allow_densify"])
        finally:
            adc.t.normal = real_normal
        after = snapshot(gs, opt)
        rec = {f"in_{k}": v for k, v in before.items()}
        rec.update({f"in_{k}": v for k, v in stats_in.items()})
        rec.update({f"out_{k}": v for k, v in after.items()})
        rec["z"] = zs[0] if zs else np.zeros((0, 3), np.float32)
        rec["counts"] = np.array([counts["cloned"], counts["split"], counts["pruned"]], np.int64)
        rec["params"] = np.array([0.00005, 0.01, 0.01, extent,
                                  -1.0 if c["max_screen"] is None else c["max_screen"],
                                  float(c["reset_opacity"]), float(c["allow_densify"]),
                                  float(c["max_gaussians"])], np.float64)
        np.savez_compressed(args.out / f"ref_adc_{name}.npz", **rec)
        print(name, n, "->", after["mu"].shape[0], dict(counts))
    return 0


if __name__ == "__main__":
    sys.exit(main())
