"""The reference's finite-difference gradient checks (tests/test_cuda_backward.py:53-263 of
the reference), re-stated against the drop-in module: same inputs, same float32 tolerances
(eps 1e-3, atol 1e-3, rtol 1e-2, nondet_tol 1e-4), calling `custom_rasterizer_cuda` and
`gaussian_splatting.rasterizer.rasterize.RasterizeFunction` exactly as the reference does.
"""

from __future__ import annotations

import pytest
import torch
from torch.autograd import gradcheck

pytestmark = pytest.mark.gpu

GRADCHECK = dict(eps=1e-3, atol=1e-3, rtol=1e-2, nondet_tol=1e-4, check_batched_grad=False,
                 raise_exception=True)


def leaf(x: torch.Tensor) -> torch.Tensor:
    return x.detach().contiguous().clone().requires_grad_(True)


def test_projection_backward_matches_finite_differences(crc, cuda_device):
    dev = cuda_device
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
            m2, c2, _ = crc.project(means.shape[0], means, quats, scales, R, t, fx, fy, cx, cy)
            ctx.save_for_backward(means, quats, scales)
            return m2, c2

        @staticmethod
        def backward(ctx, gm, gc):
            means, quats, scales = ctx.saved_tensors
            return crc.backwards_projection(gm.contiguous(), gc.contiguous(), means, quats,
                                            scales, R, t, fx, fy, cx, cy)

    m2, c2 = Project.apply(mu, q, s)
    assert torch.isfinite(m2).all() and torch.isfinite(c2).all()
    assert float(m2.detach().abs().sum()) > 1.0 and float(c2.detach().abs().sum()) > 0.1
    # cov2d reaches ~25 px^2 here; its float32 rounding (several ulp of ~2e-6 through the
    # matrix products) divided by the 2e-3 central step is ~1e-2 of finite-difference noise,
    # above atol. A 1e-2 step keeps the truncation error near 1e-4 and tests the same Jacobian.
    assert gradcheck(Project.apply, (mu, q, s), **{**GRADCHECK, "eps": 1e-2})


def test_sh_backward_matches_finite_differences(crc, cuda_device):
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
            return crc.SH(means.shape[0], cam, means, alb, coeff)

        @staticmethod
        def backward(ctx, gcol):
            means, alb, coeff = ctx.saved_tensors
            gA, gkj, gmu = crc.backwards_SH(gcol.contiguous(), means, alb, coeff, cam)
            return gmu, gA, gkj

    col = SphericalHarmonics.apply(mu, A, kj)
    assert torch.isfinite(col).all()
    assert float(col.detach().min()) > 0.05 and float(col.detach().max()) < 0.95
    assert gradcheck(SphericalHarmonics.apply, (mu, A, kj), **GRADCHECK)


def test_rasterize_backward_matches_finite_differences(crc, cuda_device):
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
            img, ids, ranges, fT, nc = crc.rasterize(n, depths, means, c2, colors, opacity, H, W)
            ctx.save_for_backward(means, c2, colors, opacity, ids, ranges, fT, nc)
            ctx.n = n
            return img

        @staticmethod
        def backward(ctx, gimg):
            means, c2, colors, opacity, ids, ranges, fT, nc = ctx.saved_tensors
            return crc.backwards_rasterization(gimg.contiguous(), means, c2, colors, opacity,
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
