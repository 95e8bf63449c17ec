"""Pins the CPU oracle before it is trusted as the checker.

* The reference's four finite-difference gradient checks (tests/test_cuda_backward.py:53-263
  of the reference: same inputs, same float32 tolerances) run against the oracle's forward
  and backward.
* Closed-form known answers for projection, binning, sorting and blending.
* Golden vectors produced by the reference's own rasterize.cu / rasterize_backward.cu on a
  B200 (tests/golden/ref_raster_*, made by tests/golden/make_golden.py).
* Golden vectors of the reference's per-Gaussian stages (project, SH, backwards_SH,
  backwards_projection) from its whole extension built against the GLM stand-in
  ("ref+shim", tests/golden/ref_gaussian_*), including the reference's quaternion gradient,
  which these tests characterise exactly (the derivative of the transposed rotation).
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch
from torch.autograd import gradcheck

GOLDEN = Path(__file__).resolve().parent / "golden"

# float32 finite differences: the reference's settings (test_cuda_backward.py:28-35)
GRADCHECK = dict(eps=1e-3, atol=1e-3, rtol=1e-2, nondet_tol=1e-4, check_batched_grad=False,
                 raise_exception=True)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().astype(np.float32)


def _leaf(x) -> torch.Tensor:
    return torch.tensor(np.asarray(x, np.float32)).clone().requires_grad_(True)


# ---- autograd wrappers around the oracle --------------------------------------------------
def oracle_project_fn(O, R, t, fx, fy, cx, cy):
    class Project(torch.autograd.Function):
        @staticmethod
        def forward(ctx, mu, q, s):
            m, c, _ = O.project(_np(mu), _np(q), _np(s), R, t, fx, fy, cx, cy)
            ctx.save_for_backward(mu, q, s)
            return torch.from_numpy(m), torch.from_numpy(c)

        @staticmethod
        def backward(ctx, gm, gc):
            mu, q, s = ctx.saved_tensors
            gmu, gq, gs = O.project_backward(_np(gm), _np(gc), _np(mu), _np(q), _np(s), R, t,
                                             fx, fy, cx, cy)
            return torch.from_numpy(gmu), torch.from_numpy(gq), torch.from_numpy(gs)

    return Project.apply


def oracle_sh_fn(O, cam):
    class SH(torch.autograd.Function):
        @staticmethod
        def forward(ctx, mu, A, kj):
            ctx.save_for_backward(mu, A, kj)
            return torch.from_numpy(O.sh(cam, _np(mu), _np(A), _np(kj)))

        @staticmethod
        def backward(ctx, g):
            mu, A, kj = ctx.saved_tensors
            gA, gkj, gmu = O.sh_backward(_np(g), _np(mu), _np(A), _np(kj), cam)
            return torch.from_numpy(gmu), torch.from_numpy(gA), torch.from_numpy(gkj)

    return SH.apply


def oracle_raster_fn(O, depths, H, W):
    class Raster(torch.autograd.Function):
        @staticmethod
        def forward(ctx, mean, cov, rgb, op):
            out = O.rasterize(depths, _np(mean), _np(cov), _np(rgb), _np(op).reshape(-1), H, W)
            ctx.save_for_backward(mean, cov, rgb, op)
            ctx.out = out
            return torch.from_numpy(out["img"])

        @staticmethod
        def backward(ctx, g):
            mean, cov, rgb, op = ctx.saved_tensors
            o = ctx.out
            gm, gc, gcol, ga, _ = O.rasterize_backward(
                _np(g), _np(mean), _np(cov), _np(rgb), _np(op).reshape(-1), o["sorted_ids"],
                o["tile_ranges"], o["final_T"], o["n_contrib"], H, W)
            return (torch.from_numpy(gm), torch.from_numpy(gc), torch.from_numpy(gcol),
                    torch.from_numpy(ga).view_as(op))

    return Raster.apply


def oracle_pipeline_fn(O, R, t, fx, fy, cx, cy, H, W):
    cam = O.camera_position(R, t)

    class Pipeline(torch.autograd.Function):
        @staticmethod
        def forward(ctx, mu, q, s, op, A, kj):
            out = O.render(_np(mu), _np(q), _np(s), _np(op), _np(A), _np(kj), R, t, fx, fy, cx,
                           cy, H, W)
            ctx.save_for_backward(mu, q, s, op, A, kj)
            ctx.out = out
            return torch.from_numpy(out["img"])

        @staticmethod
        def backward(ctx, g):
            mu, q, s, op, A, kj = ctx.saved_tensors
            o = ctx.out
            gm, gc, gcol, ga, _ = O.rasterize_backward(
                _np(g), o["mean2d"], o["cov2d"], o["colors"], _np(op).reshape(-1),
                o["sorted_ids"], o["tile_ranges"], o["final_T"], o["n_contrib"], H, W)
            gA, gkj, gmu_sh = O.sh_backward(gcol, _np(mu), _np(A), _np(kj), cam)
            gmu, gq, gs = O.project_backward(gm, gc, _np(mu), _np(q), _np(s), R, t, fx, fy, cx,
                                             cy)
            return (torch.from_numpy(gmu + gmu_sh), torch.from_numpy(gq), torch.from_numpy(gs),
                    torch.from_numpy(ga).view_as(op), torch.from_numpy(gA),
                    torch.from_numpy(gkj))

    return Pipeline.apply


# ---- the reference's four gradient checks, on the oracle ------------------------------------
def test_oracle_projection_gradcheck(oracle):
    R, t = np.eye(3, dtype=np.float32), np.zeros(3, np.float32)
    fn = oracle_project_fn(oracle, R, t, 200.0, 200.0, 100.0, 100.0)
    mu = _leaf([[0.30, -0.20, 3.5], [-0.25, 0.15, 5.0]])
    quat = np.array([1.0, 0.15, -0.05, 0.02], np.float32)
    quat /= np.linalg.norm(quat)
    q = _leaf(np.tile(quat, (2, 1)))
    s = _leaf([[-2.2, -2.0, -1.8], [-2.5, -2.1, -2.3]])
    m, c = fn(mu, q, s)
    assert float(m.detach().abs().sum()) > 1.0 and float(c.detach().abs().sum()) > 0.1
    # cov2d reaches ~25 px^2 here, where one float32 ulp (~2e-6) over the 2e-3 central step
    # is ~1e-3 of noise, the size of atol; a 1e-2 step keeps the truncation error ~1e-4.
    assert gradcheck(fn, (mu, q, s), **{**GRADCHECK, "eps": 1e-2})


def test_oracle_sh_gradcheck(oracle):
    cam = np.zeros(3, np.float32)
    fn = oracle_sh_fn(oracle, cam)
    mu = _leaf([[0.40, -0.30, 2.5], [-0.20, 0.50, 3.0]])
    A = _leaf(np.zeros((2, 3)))
    kj = _leaf(np.linspace(-0.005, 0.005, 90, dtype=np.float32).reshape(2, 15, 3))
    col = fn(mu, A, kj)
    assert 0.05 < float(col.detach().min()) and float(col.detach().max()) < 0.95
    assert gradcheck(fn, (mu, A, kj), **GRADCHECK)


def test_oracle_rasterize_gradcheck(oracle):
    fn = oracle_raster_fn(oracle, np.array([2.0], np.float32), 16, 16)
    mean = _leaf([[8.0, 8.0]])
    cov = _leaf([[4.0, 0.0, 4.0]])
    rgb = _leaf([[0.25, 0.45, 0.70]])
    op = _leaf([[0.6]])

    def center(mean, cov, rgb, op):
        return fn(mean, cov, rgb, op)[6:10, 6:10].sum()

    assert float(center(mean, cov, rgb, op).detach()) > 1e-2
    assert gradcheck(center, (mean, cov, rgb, op), **GRADCHECK)


def test_oracle_full_pipeline_gradcheck(oracle):
    R, t = np.eye(3, dtype=np.float32), np.zeros(3, np.float32)
    fn = oracle_pipeline_fn(oracle, R, t, 16.0, 16.0, 8.0, 8.0, 16, 16)
    mu = _leaf([[0.05, -0.04, 4.0]])
    quat = np.array([1.0, 0.1, -0.05, 0.02], np.float32)
    quat /= np.linalg.norm(quat)
    q = _leaf(quat.reshape(1, 4))
    s = _leaf(np.full((1, 3), -2.0))
    op = _leaf([[0.5]])
    A = _leaf(np.zeros((1, 3)))
    kj = _leaf(np.linspace(-0.005, 0.005, 45, dtype=np.float32).reshape(1, 15, 3))

    def center(*args):
        return fn(*args)[7:9, 7:9].sum()

    assert float(center(mu, q, s, op, A, kj).detach()) > 1e-3
    assert gradcheck(center, (mu, q, s, op, A, kj), **GRADCHECK)


# ---- closed-form known answers --------------------------------------------------------------
def test_projection_closed_form(oracle):
    """Identity rotation and camera: Sigma = diag(e^{2s}), cov2d = J Sigma J^T + 0.3 I."""
    mu = np.array([[0.5, -0.25, 4.0], [0.0, 0.0, 0.1]], np.float32)  # second one is culled
    q = np.array([[1, 0, 0, 0], [1, 0, 0, 0]], np.float32)
    s = np.array([[-2.0, -1.5, -1.0], [0, 0, 0]], np.float32)
    fx, fy, cx, cy = 300.0, 200.0, 64.0, 32.0
    m, c, d = oracle.project(mu, q, s, np.eye(3), np.zeros(3), fx, fy, cx, cy)
    x, y, z = (float(v) for v in mu[0])
    sig = np.exp(2.0 * s[0].astype(np.float64))
    J = np.array([[fx / z, 0, -fx * x / z**2], [0, fy / z, -fy * y / z**2]])
    C = J @ np.diag(sig) @ J.T
    np.testing.assert_allclose(m[0], [fx * x / z + cx, fy * y / z + cy], rtol=1e-6)
    np.testing.assert_allclose(c[0], [C[0, 0] + 0.3, C[0, 1], C[1, 1] + 0.3], rtol=1e-5)
    assert d[0] == np.float32(4.0)
    assert not m[1].any() and not c[1].any() and d[1] == 0.0  # z <= 0.2: zeros


def test_projection_quaternion_is_normalised(oracle):
    mu = np.array([[0.1, 0.2, 3.0]] * 2, np.float32)
    q = np.array([[0.9, 0.3, -0.2, 0.1], [1.8, 0.6, -0.4, 0.2]], np.float32)  # same rotation
    s = np.array([[-2.0, -1.0, -3.0]] * 2, np.float32)
    _, c, _ = oracle.project(mu, q, s, np.eye(3), np.zeros(3), 100.0, 100.0, 0.0, 0.0)
    np.testing.assert_allclose(c[0], c[1], rtol=2e-6)


def test_binning_known_answer(oracle):
    """A circular splat of covariance 4 px^2 at (40.5, 20.5) in a 64x48 image: 3-sigma radius
    ceil(3*sqrt(4.3)) = 7 px, pixel box [33, 48) x [13, 28) -> tiles x 2..2, y 0..1."""
    mean = np.array([[40.5, 20.5]], np.float32)
    cov = np.array([[4.0, 0.0, 4.0]], np.float32)
    M, counts = oracle.count(mean, cov, 48, 64)
    assert M == 2 and counts.tolist() == [2]
    keys, ids, ranges = oracle.bin(mean, cov, np.array([3.0], np.float32), 48, 64)
    tiles = (keys >> np.uint64(32)).astype(np.int64).tolist()
    assert tiles == [2, 6] and ids.tolist() == [0, 0]
    assert ranges.tolist()[2] == [0, 1] and ranges.tolist()[6] == [1, 2]
    assert sum(r[1] - r[0] for r in ranges.tolist()) == 2


def test_sort_is_stable_on_equal_depths(oracle):
    """Equal (tile, depth) keys keep Gaussian-index order; nearer depth sorts first."""
    mean = np.array([[8, 8], [8, 8], [8, 8], [8, 8]], np.float32)
    cov = np.array([[2, 0, 2]] * 4, np.float32)
    depths = np.array([5.0, 3.0, 5.0, 3.0], np.float32)
    _, ids, ranges = oracle.bin(mean, cov, depths, 16, 16)
    assert ids.tolist() == [1, 3, 0, 2] and ranges.tolist() == [[0, 4]]


def test_degenerate_covariance_is_skipped(oracle):
    mean = np.array([[8, 8], [8, 8]], np.float32)
    cov = np.array([[1, 1, 1], [1, 2, 1]], np.float32)  # det 0 and det < 0
    M, counts = oracle.count(mean, cov, 16, 16)
    assert M == 0 and counts.tolist() == [0, 0]


def test_blend_single_splat_closed_form(oracle):
    """At the splat centre power = 0, so alpha = opacity; one splat gives C = c * o."""
    mean = np.array([[5.0, 6.0]], np.float32)
    cov = np.array([[3.0, 0.5, 2.0]], np.float32)
    col = np.array([[0.2, 0.4, 0.8]], np.float32)
    op = np.array([0.7], np.float32)
    out = oracle.rasterize(np.array([1.0], np.float32), mean, cov, col, op, 16, 16)
    np.testing.assert_allclose(out["img"][6, 5], col[0] * 0.7, rtol=1e-6)
    assert out["final_T"][6, 5] == np.float32(1.0) - np.float32(0.7)
    assert out["n_contrib"][6, 5] == 1
    assert out["n_contrib"][0, 15] == 0 and out["final_T"][0, 15] == 1.0


def test_blend_stops_below_transmittance_floor(oracle):
    """Opaque splats (alpha = 0.99) stacked at one pixel: T = 0.01^k stops after 2."""
    n = 5
    mean = np.tile(np.array([[4.0, 4.0]], np.float32), (n, 1))
    cov = np.tile(np.array([[2.0, 0.0, 2.0]], np.float32), (n, 1))
    col = np.tile(np.array([[1.0, 1.0, 1.0]], np.float32), (n, 1))
    op = np.ones(n, np.float32)
    depths = np.arange(1, n + 1, dtype=np.float32)
    out = oracle.rasterize(depths, mean, cov, col, op, 16, 16)
    assert out["n_contrib"][4, 4] == 2
    assert out["final_T"][4, 4] < 1e-4


def test_empty_image_when_nothing_visible(oracle):
    mean = np.array([[-100.0, -100.0]], np.float32)
    cov = np.array([[4.0, 0.0, 4.0]], np.float32)
    out = oracle.rasterize(np.array([1.0], np.float32), mean, cov, np.ones((1, 3), np.float32),
                           np.ones(1, np.float32), 20, 30)
    assert len(out["sorted_ids"]) == 0 and not out["img"].any()
    assert (out["final_T"] == 1).all() and not out["tile_ranges"].any()


# ---- golden vectors from the reference's own kernels ----------------------------------------
def golden_files() -> list[Path]:
    return sorted(GOLDEN.glob("ref_raster_*.npz"))


@pytest.mark.parametrize("path", golden_files(), ids=lambda p: p.stem)
def test_oracle_matches_reference_golden(oracle, path):
    """Binning is bit-exact; blending matches within float tolerance on every pixel whose
    threshold decisions the oracle does not flag as ambiguous; gradients within 1e-4."""
    g = dict(np.load(path))
    H, W = int(g["H"]), int(g["W"])
    out = oracle.rasterize(g["depths"], g["mean2d"], g["cov2d"], g["colors"], g["alpha"], H, W)
    np.testing.assert_array_equal(out["sorted_ids"], g["sorted_ids"])
    np.testing.assert_array_equal(out["tile_ranges"], g["tile_ranges"])
    ok = ~out["ambiguous"]
    assert ok.mean() > 0.99
    np.testing.assert_array_equal(out["n_contrib"][ok], g["n_contrib"][ok])
    np.testing.assert_allclose(out["final_T"][ok], g["final_T"][ok], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(out["img"][ok], g["img"][ok], rtol=1e-4, atol=1e-5)
    gm, gc, gcol, ga, amb = oracle.rasterize_backward(
        g["grad_img"], g["mean2d"], g["cov2d"], g["colors"], g["alpha"], g["sorted_ids"],
        g["tile_ranges"], g["final_T"], g["n_contrib"], H, W)
    keep = ~amb
    for mine, ref in ((gm, g["g_mean2d"]), (gc, g["g_cov2d"]), (gcol, g["g_colors"]),
                      (ga.reshape(-1), g["g_alpha"].reshape(-1))):
        scale = float(np.abs(ref).max()) + 1e-12
        np.testing.assert_allclose(mine[keep], ref[keep], rtol=1e-3, atol=2e-5 * scale)


# ---- golden vectors of the reference's per-Gaussian stages (ref+shim) -----------------------
def gaussian_golden_files() -> list[Path]:
    return sorted(GOLDEN.glob("ref_gaussian_*.npz"))


def grad_band(a, b, rtol=1e-4):
    """(fraction of elements outside rtol * (|b| + rms(b)), worst error / band)."""
    b = np.asarray(b, np.float64)
    a = np.asarray(a, np.float64).reshape(b.shape)
    rms = float(np.sqrt(np.mean(b * b))) if b.size else 0.0
    band = rtol * (np.abs(b) + rms) + 1e-30
    err = np.abs(a - b)
    return float((err > band).mean()), float((err / band).max())


def _gaussian_golden(path):
    g = dict(np.load(path))
    fx, fy, cx, cy = (float(v) for v in g["intr"])
    return g, (fx, fy, cx, cy)


@pytest.mark.parametrize("path", gaussian_golden_files(), ids=lambda p: p.stem)
def test_oracle_projection_and_sh_match_reference_golden(oracle, path):
    """Screen means and depths bit-exact; 2D covariance within 1e-5 of its own scale (the
    oracle's fused multiply-adds approximate nvcc's contraction); colours within 1e-5 / 1e-6."""
    g, (fx, fy, cx, cy) = _gaussian_golden(path)
    m, c, d = oracle.project(g["mu"], g["q"], g["s"], g["R"], g["t"], fx, fy, cx, cy)
    np.testing.assert_array_equal(m, g["mean2d"])
    np.testing.assert_array_equal(d, g["depths"])
    assert ((d == 0) == (g["depths"] == 0)).all()
    scale = np.maximum(np.abs(g["cov2d"][:, [0]]), np.abs(g["cov2d"][:, [2]]))
    assert (np.abs(c.astype(np.float64) - g["cov2d"]) <= 1e-5 * scale + 1e-6).all()
    col = oracle.sh(g["cam"], g["mu"], g["A"], g["k_j"])
    np.testing.assert_allclose(col, g["colors"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("path", gaussian_golden_files(), ids=lambda p: p.stem)
def test_oracle_sh_backward_matches_reference_golden(oracle, path):
    g, _ = _gaussian_golden(path)
    gA, gkj, gmu = oracle.sh_backward(g["g_colors"], g["mu"], g["A"], g["k_j"], g["cam"])
    np.testing.assert_array_equal(gA, g["g_A"])
    for mine, key in ((gkj, "g_k_j"), (gmu, "g_mu_sh")):
        out, worst = grad_band(mine, g[key])
        assert out == 0.0, (key, out, worst)


@pytest.mark.parametrize("path", gaussian_golden_files(), ids=lambda p: p.stem)
def test_oracle_projection_backward_against_reference_golden(oracle, path):
    """Mean and log-scale gradients within 1e-4 of the reference's. The quaternion gradient is
    where the two differ on purpose: the reference's (golden) equals the float64 derivative of
    the TRANSPOSED rotation to within 1e-4 of the band, and misses the true derivative of its
    own forward on most elements; the oracle's equals the true derivative."""
    from tests.proj64 import projection_grads64, transposed_rotation_q_grad64

    g, (fx, fy, cx, cy) = _gaussian_golden(path)
    args = (g["g_mean2d"], g["g_cov2d"], g["mu"], g["q"], g["s"], g["R"], g["t"], fx, fy, cx, cy)
    omu, oq, os_ = oracle.project_backward(*args)
    for mine, key in ((omu, "g_mu"), (os_, "g_s")):
        out, worst = grad_band(mine, g[key])
        assert out == 0.0, (key, out, worst)
    live = np.linalg.norm(g["q"], axis=1) > 0  # d/dq is undefined at the zero quaternion
    visible = g["depths"] > 0
    rows = live & visible
    true_q = projection_grads64(*args)[1].numpy()
    transposed_q = transposed_rotation_q_grad64(*args).numpy()
    assert grad_band(oq[rows], true_q[rows])[0] == 0.0
    assert grad_band(g["g_q"][rows], transposed_q[rows])[0] == 0.0
    assert grad_band(g["g_q"][rows], true_q[rows])[0] > 0.5
