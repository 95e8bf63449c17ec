"""Device adaptive density control (gs_adc_plan / gs_adc_apply behind the reference-API
`gaussian_splatting.utils.adc.adaptive_density_control`) against the reference's own
results on the golden cases (tests/golden/ref_adc_*.npz, fed the same split normals) and
against the numpy oracle (oracle/adc_oracle.py) on a larger seeded scene.

Counts are exact; kept parameters and every Adam moment are bit-exact; the split children's
means and log-scales agree within float32 rounding (rtol 1e-5, atol 1e-6: the device's
expf/logf and fused multiply-adds against the CPU's)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from test_adc_oracle import NAMES, golden_cases, load_case

pytestmark = pytest.mark.gpu

GROUPS = ("mu", "q", "Scale", "Opacity", "Albedo Coefficient", "Illumination Coefficients")


def make_state(dev, params, m, v, step, grad_accum, denom, radii):
    """Gaussians and a torch Adam with the reference's six named groups and given moments."""
    from gaussian_splatting.scene.gaussian import gaussian

    n = params["mu"].shape[0]
    gs = gaussian(n)
    groups = []
    for name, grp in zip(NAMES, GROUPS):
        p = torch.nn.Parameter(torch.from_numpy(np.ascontiguousarray(params[name])).to(dev))
        setattr(gs, name, p)
        groups.append({"params": [p], "lr": 1e-3, "name": grp})
    opt = torch.optim.Adam(groups, lr=0.01, eps=1e-15)
    for name in NAMES:
        p = getattr(gs, name)
        opt.state[p] = {"step": torch.tensor(float(step)),
                        "exp_avg": torch.from_numpy(m[name]).to(dev),
                        "exp_avg_sq": torch.from_numpy(v[name]).to(dev)}
    gs.xyz_grad_accum = torch.from_numpy(grad_accum).to(dev)
    gs.denom = torch.from_numpy(denom).to(dev)
    gs.max_radii2D = torch.from_numpy(radii).to(dev)
    return gs, opt


def group_state(opt, name):
    grp = next(g for g in opt.param_groups if g["name"] == GROUPS[NAMES.index(name)])
    p = grp["params"][0]
    return p, opt.state[p]


def check_outputs(gs, opt, ref_p, ref_m, ref_v, n_split):
    n_out = ref_p["mu"].shape[0]
    assert gs.N == n_out
    for name in NAMES:
        p, st = group_state(opt, name)
        assert p is getattr(gs, name), name
        mine = p.detach().cpu().numpy()
        assert mine.shape == ref_p[name].shape, name
        if name in ("mu", "s") and n_split:
            np.testing.assert_allclose(mine, ref_p[name], rtol=1e-5, atol=1e-6, err_msg=name)
        else:
            np.testing.assert_array_equal(mine, ref_p[name], err_msg=name)
        np.testing.assert_array_equal(st["exp_avg"].cpu().numpy(), ref_m[name],
                                      err_msg=name + " exp_avg")
        np.testing.assert_array_equal(st["exp_avg_sq"].cpu().numpy(), ref_v[name],
                                      err_msg=name + " exp_avg_sq")
    assert gs.xyz_grad_accum.shape == (n_out, 1) and not gs.xyz_grad_accum.any()
    assert gs.denom.shape == (n_out, 1) and not gs.denom.any()
    assert gs.max_radii2D.shape == (n_out,) and not gs.max_radii2D.any()


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_device_adc_matches_reference(cuda_device, path):
    from gaussian_splatting.utils.adc import adaptive_density_control

    d, params, m, v, kw = load_case(path)
    gs, opt = make_state(cuda_device, params, m, v, d["in_mu_step"], d["in_grad_accum"],
                         d["in_denom"], d["in_max_radii"])
    z = torch.from_numpy(d["z"]).to(cuda_device)
    gs, opt, stats = adaptive_density_control(gs, opt, split_normals=z, **kw)
    torch.cuda.synchronize()
    assert [stats["cloned"], stats["split"], stats["pruned"]] == list(d["counts"])
    check_outputs(gs, opt, {n: d[f"out_{n}"] for n in NAMES},
                  {n: d[f"out_{n}_exp_avg"] for n in NAMES},
                  {n: d[f"out_{n}_exp_avg_sq"] for n in NAMES}, int(d["counts"][1]))
    for name in NAMES:
        assert float(group_state(opt, name)[1]["step"]) == float(d[f"out_{name}_step"])


def random_scene(n, seed):
    g = np.random.default_rng(seed)
    f = np.float32
    q = g.standard_normal((n, 4)).astype(f)
    params = {"mu": (g.random((n, 3)) * 4 - 2).astype(f),
              "q": (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(f),
              "s": (g.standard_normal((n, 3)) * 1.2 + math.log(0.04)).astype(f),
              "alpha": (g.standard_normal((n, 1)) * 3.0).astype(f),
              "A": (g.standard_normal((n, 3)) * 0.5).astype(f),
              "k_j": (g.standard_normal((n, 15, 3)) * 0.05).astype(f)}
    m = {k: (g.standard_normal(p.shape) * 1e-3).astype(f) for k, p in params.items()}
    v = {k: (g.random(p.shape) * 1e-5).astype(f) for k, p in params.items()}
    stats = ((g.random((n, 1)) * 4e-4).astype(f), g.integers(0, 5, (n, 1)).astype(f),
             (g.random(n) * 40.0).astype(f))
    return params, m, v, stats


@pytest.mark.parametrize("reset", [False, True])
def test_device_adc_matches_oracle_large(cuda_device, reset):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from gaussian_splatting.utils.adc import adaptive_density_control
    from oracle import adc_oracle

    n = 120_000
    params, m, v, (ga, de, ra) = random_scene(n, 7 + int(reset))
    kw = dict(grad_threshold=0.00005, percent_dense=0.01, min_opacity=0.01, scene_extent=4.0,
              max_screen_size=20.0, reset_opacity=reset, max_gaussians=800_000)
    clone, split, *_ = adc_oracle.classify(
        params["s"], params["alpha"], ga, de, ra, grad_threshold=0.00005, percent_dense=0.01,
        scene_extent=4.0, min_opacity=0.01, max_screen_size=20.0, densify=True, prune=True)
    n_split = int(split.sum())
    z = np.random.default_rng(99).standard_normal((2 * n_split, 3)).astype(np.float32)
    ref_p, ref_m, ref_v, counts = adc_oracle.adaptive_density_control(
        params, m, v, ga, de, ra, z, **kw)
    assert n_split > 1000 and counts[0] > 1000 and counts[2] > 1000

    gs, opt = make_state(cuda_device, params, m, v, 7, ga, de, ra)
    gs, opt, stats = adaptive_density_control(
        gs, opt, split_normals=torch.from_numpy(z).to(cuda_device), **kw)
    assert (stats["cloned"], stats["split"], stats["pruned"]) == counts
    check_outputs(gs, opt, ref_p, ref_m, ref_v, n_split)


def test_device_adc_no_densify_and_optimizer_steps(cuda_device):
    """allow_densify=False leaves the set untouched and only resets the statistics; after a
    densifying call the optimizer still steps over the new tensors."""
    from gaussian_splatting.utils.adc import adaptive_density_control

    params, m, v, (ga, de, ra) = random_scene(5000, 3)
    gs, opt = make_state(cuda_device, params, m, v, 3, ga, de, ra)
    gs, opt, stats = adaptive_density_control(gs, opt, scene_extent=4.0, allow_densify=False)
    assert stats == {"cloned": 0, "split": 0, "pruned": 0}
    np.testing.assert_array_equal(gs.mu.detach().cpu().numpy(), params["mu"])
    assert not gs.denom.any()

    gs.xyz_grad_accum = torch.from_numpy(ga).to(cuda_device)
    gs.denom = torch.from_numpy(de).to(cuda_device)
    gs, opt, stats = adaptive_density_control(gs, opt, scene_extent=4.0, max_screen_size=20.0)
    assert stats["split"] > 0 and stats["cloned"] > 0
    for name in NAMES:
        p = getattr(gs, name)
        p.grad = torch.ones_like(p)
    opt.step()
    for name in NAMES:
        p, st = group_state(opt, name)
        assert st["exp_avg"].shape == p.shape and torch.isfinite(p).all()


def test_densification_statistics_helpers(cuda_device):
    """accumulate_densification_stats (one gs_densify_stats launch) against the reference
    helper's semantics (gaussian_splatting/utils/adc.py:58-80), restated with torch ops: the
    norm of the screen-space mean gradient scaled by (W/2, H/2) added where it is non-zero,
    counted in denom; with buffers grown from a shorter set (prefix kept, new rows zero), a
    [N, 3] gradient (only the first two columns used) and no image size (scale 1)."""
    from gaussian_splatting.scene.gaussian import gaussian
    from gaussian_splatting.utils.adc import (accumulate_densification_stats,
                                              ensure_densification_state, update_max_radii2d)

    dev = cuda_device
    g = torch.Generator("cpu").manual_seed(21)
    n = 5000
    gs = gaussian(n)
    gs.mu = torch.randn(n, 3, generator=g).to(dev)
    gs.xyz_grad_accum = torch.rand(n - 100, 1, generator=g).to(dev)
    gs.denom = torch.full((n - 100, 1), 2.0).to(dev)
    gs.max_radii2D = torch.rand(n - 100, generator=g).to(dev)
    ensure_densification_state(gs)
    assert gs.xyz_grad_accum.shape == (n, 1) and gs.max_radii2D.shape == (n,)
    assert float(gs.xyz_grad_accum[n - 100:].abs().sum()) == 0.0
    acc, den = gs.xyz_grad_accum.clone(), gs.denom.clone()
    grad = torch.randn(n, 3, generator=g)
    grad[::7] = 0.0  # not visible in this view
    grad = grad.to(dev)
    for width, height in ((1920, 1080), (None, None)):
        accumulate_densification_stats(gs, grad, width=width, height=height)
        scale = torch.tensor([width / 2.0, height / 2.0] if width else [1.0, 1.0], device=dev)
        norm = torch.norm(grad[:, :2] * scale, dim=-1, keepdim=True)
        vis = norm.squeeze(-1) > 0
        acc[vis] += norm[vis]
        den[vis] += 1.0
        torch.testing.assert_close(gs.xyz_grad_accum, acc, rtol=1e-6, atol=0)
        assert torch.equal(gs.denom, den)
    radii = torch.rand(n, generator=g).to(dev)
    before = gs.max_radii2D.clone()
    update_max_radii2d(gs, radii)
    assert torch.equal(gs.max_radii2D, torch.maximum(before, radii))
