"""The reference's finite-difference gradient checks (tests/test_cuda_backward.py:53-263 of the
reference), run against this library's drop-in module AND against the reference's own build
(the whole extension compiled against the GLM stand-in by oracle/build_ref.py, "ref+shim").

The SH, blend and full-pipeline checks use the reference's settings unchanged: eps 1e-3,
atol 1e-3, rtol 1e-2, nondet_tol 1e-4. The projection check is where the settings matter,
measured on a B200 against both builds:
* As shipped (eps 1e-3) the reference's own build fails it. Its log-scale gradient is correct
  (float64 autograd agrees to 1e-4), yet it misses the float32 finite difference by more than
  atol: cov2d reaches about 25 px^2, so float32 rounding over the 2e-3 central step is about
  1e-2 of noise (e.g. 9.76e-3 analytic against 8.58e-3 numeric). This library fails the same
  way at eps 1e-3, on log-scales and quaternions.
* At eps 1e-2 (truncation error near 1e-4) this library passes for means, quaternions and
  log-scales; the reference's build passes for means and log-scales and still fails for the
  quaternion, whose gradient it computes as the derivative of the transposed rotation
  (tests/test_oracle_kat.py characterises it exactly).
So this library's projection check runs at eps 1e-2, and the reference's results above are
asserted as recorded facts.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
from torch.autograd import gradcheck
from torch.autograd.gradcheck import GradcheckError

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
GRADCHECK = dict(eps=1e-3, atol=1e-3, rtol=1e-2, nondet_tol=1e-4, check_batched_grad=False,
                 raise_exception=True)


def leaf(x: torch.Tensor) -> torch.Tensor:
    return x.detach().contiguous().clone().requires_grad_(True)


def _ref_full():
    p = str(ROOT / "oracle" / "_ref" / "ref_full")
    if p not in sys.path:
        sys.path.insert(0, p)
    try:
        import ref_full
    except ImportError:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    return ref_full


@pytest.fixture(params=["ours", "reference"])
def module(request, crc):
    return crc if request.param == "ours" else _ref_full()


def _projection_setup(mod, dev):
    R = torch.eye(3, device=dev)
    t = torch.zeros(3, device=dev)
    fx = fy = 200.0
    cx = cy = 100.0
    mu = leaf(torch.tensor([[0.30, -0.20, 3.5], [-0.25, 0.15, 5.0]], device=dev))
    quat = torch.tensor([1.0, 0.15, -0.05, 0.02], device=dev)
    q = leaf((quat / quat.norm()).expand(2, 4))
    s = leaf(torch.tensor([[-2.2, -2.0, -1.8], [-2.5, -2.1, -2.3]], device=dev))

    class Project(torch.autograd.Function):
        @staticmethod
        def forward(ctx, means, quats, scales):
            means, quats, scales = means.contiguous(), quats.contiguous(), scales.contiguous()
            m2, c2, _ = mod.project(means.shape[0], means, quats, scales, R, t, fx, fy, cx, cy)
            ctx.save_for_backward(means, quats, scales)
            return m2, c2

        @staticmethod
        def backward(ctx, gm, gc):
            means, quats, scales = ctx.saved_tensors
            return mod.backwards_projection(gm.contiguous(), gc.contiguous(), means, quats,
                                            scales, R, t, fx, fy, cx, cy)

    return Project.apply, (mu, q, s)


def _only(fn, inputs, k):
    """fn as a function of input k alone (the others held fixed)."""
    fixed = [x.detach() for x in inputs]

    def f(x):
        args = list(fixed)
        args[k] = x
        return fn(*args)

    return f, (leaf(inputs[k]),)


def test_projection_backward_matches_finite_differences(crc, cuda_device):
    fn, inputs = _projection_setup(crc, cuda_device)
    m2, c2 = fn(*inputs)
    assert torch.isfinite(m2).all() and torch.isfinite(c2).all()
    assert float(m2.detach().abs().sum()) > 1.0 and float(c2.detach().abs().sum()) > 0.1
    assert gradcheck(fn, inputs, **{**GRADCHECK, "eps": 1e-2})


def test_reference_build_fails_its_projection_check_as_shipped(cuda_device):
    """The reference's projection check, exactly as shipped, fails on the reference's own
    build (float32 finite-difference noise at eps 1e-3, and the quaternion gradient)."""
    fn, inputs = _projection_setup(_ref_full(), cuda_device)
    with pytest.raises(GradcheckError):
        gradcheck(fn, inputs, **GRADCHECK)


def test_reference_build_quaternion_gradient_fails_at_eps_1e2(cuda_device):
    """At eps 1e-2 the reference's means and log-scales pass and its quaternion fails."""
    fn, inputs = _projection_setup(_ref_full(), cuda_device)
    G = {**GRADCHECK, "eps": 1e-2}
    for k in (0, 2):
        f, x = _only(fn, inputs, k)
        assert gradcheck(f, x, **G)
    f, x = _only(fn, inputs, 1)
    with pytest.raises(GradcheckError):
        gradcheck(f, x, **G)


def test_sh_backward_matches_finite_differences(module, cuda_device):
    dev = cuda_device
    cam = torch.zeros(3, device=dev)
    mu = leaf(torch.tensor([[0.40, -0.30, 2.5], [-0.20, 0.50, 3.0]], device=dev))
    A = leaf(torch.zeros(2, 3, device=dev))
    kj = leaf(torch.linspace(-0.005, 0.005, 90, device=dev).reshape(2, 15, 3))

    class SphericalHarmonics(torch.autograd.Function):
        @staticmethod
        def forward(ctx, means, alb, coeff):
            means, alb, coeff = means.contiguous(), alb.contiguous(), coeff.contiguous()
            ctx.save_for_backward(means, alb, coeff)
            return module.SH(means.shape[0], cam, means, alb, coeff)

        @staticmethod
        def backward(ctx, gcol):
            means, alb, coeff = ctx.saved_tensors
            gA, gkj, gmu = module.backwards_SH(gcol.contiguous(), means, alb, coeff, cam)
            return gmu, gA, gkj

    col = SphericalHarmonics.apply(mu, A, kj)
    assert torch.isfinite(col).all()
    assert float(col.detach().min()) > 0.05 and float(col.detach().max()) < 0.95
    assert gradcheck(SphericalHarmonics.apply, (mu, A, kj), **GRADCHECK)


def test_rasterize_backward_matches_finite_differences(module, cuda_device):
    dev = cuda_device
    H = W = 16
    mean = leaf(torch.tensor([[8.0, 8.0]], device=dev))
    cov = leaf(torch.tensor([[4.0, 0.0, 4.0]], device=dev))
    rgb = leaf(torch.tensor([[0.25, 0.45, 0.70]], device=dev))
    op = leaf(torch.tensor([[0.6]], device=dev))
    depths = torch.tensor([2.0], device=dev)

    class Raster(torch.autograd.Function):
        @staticmethod
        def forward(ctx, means, c2, colors, opacity):
            n = means.shape[0]
            means, c2 = means.contiguous(), c2.contiguous()
            colors, opacity = colors.contiguous(), opacity.contiguous()
            img, ids, ranges, fT, nc = module.rasterize(n, depths, means, c2, colors, opacity, H, W)
            ctx.save_for_backward(means, c2, colors, opacity, ids, ranges, fT, nc)
            ctx.n = n
            return img

        @staticmethod
        def backward(ctx, gimg):
            means, c2, colors, opacity, ids, ranges, fT, nc = ctx.saved_tensors
            return module.backwards_rasterization(gimg.contiguous(), means, c2, colors, opacity,
                                                  ids, ranges, fT, nc, ctx.n, H, W)

    def centre(m, c, r, o):
        return Raster.apply(m, c, r, o)[6:10, 6:10].sum()

    val = centre(mean, cov, rgb, op)
    assert torch.isfinite(val) and float(val.detach()) > 1e-2
    assert gradcheck(centre, (mean, cov, rgb, op), **GRADCHECK)


def test_full_pipeline_backward_matches_finite_differences(cuda_device):
    from gaussian_splatting.rasterizer.rasterize import RasterizeFunction

    dev = cuda_device
    H = W = 16
    R = torch.eye(3, device=dev)
    t = torch.zeros(3, device=dev)
    mu = leaf(torch.tensor([[0.05, -0.04, 4.0]], device=dev))
    quat = torch.tensor([1.0, 0.1, -0.05, 0.02], device=dev)
    q = leaf((quat / quat.norm()).reshape(1, 4))
    s = leaf(torch.full((1, 3), -2.0, device=dev))
    op = leaf(torch.tensor([[0.5]], device=dev))
    A = leaf(torch.zeros(1, 3, device=dev))
    kj = leaf(torch.linspace(-0.005, 0.005, 45, device=dev).reshape(1, 15, 3))

    def pipeline(m, qq, ss, o, a, k):
        img = RasterizeFunction.apply(m, qq, ss, o, a, k, R, t, 16.0, 16.0, 8.0, 8.0, H, W)
        return img[7:9, 7:9].sum()

    val = pipeline(mu, q, s, op, A, kj)
    assert torch.isfinite(val) and float(val.detach()) > 1e-3
    assert gradcheck(pipeline, (mu, q, s, op, A, kj), **GRADCHECK)
