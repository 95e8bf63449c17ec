"""Autograd wrapper of the rasterizer, API-identical to the reference's
gaussian_splatting/rasterizer/rasterize.py:9-160.

`RasterizeFunction.apply(mu, q, s, alpha, albedo, k_j, cam_rotation, cam_translation,
fx, fy, cx, cy, height, width)` renders an [H, W, 3] image; `alpha` is opacity in (0, 1).
Class attributes, as in the reference:
* `last_radii2d`  (N,) screen radii 3*sqrt(max(mid + sqrt(max(((a-c)/2)^2 + b^2, 0.1)), 0))
  of the last forward (rasterize.py:49-53 of the reference);
* `last_mean2d_grad` (N, 2) dL/dmean2d of the last backward, for densification.
`rasterize(gaussians, view)` applies the sigmoid to the opacity logits first.
"""

from __future__ import annotations

import torch as t

from gaussian_splatting.scene.gaussian import gaussian

try:
    import custom_rasterizer_cuda as crc
except ImportError:  # surfaced at first use, as in the reference
    crc = None


def _screen_radii(cov_2d: t.Tensor) -> t.Tensor:
    a, b, c = cov_2d[:, 0], cov_2d[:, 1], cov_2d[:, 2]
    mid = 0.5 * (a + c)
    radius = mid + t.sqrt(t.clamp((0.5 * (a - c)) ** 2 + b * b, min=0.1))
    return (3.0 * t.sqrt(t.clamp(radius, min=0.0))).detach()


class RasterizeFunction(t.autograd.Function):
    """Projection -> SH colour -> tile binning/sort -> alpha blend, and the reverse."""

    last_mean2d_grad: t.Tensor | None = None
    last_radii2d: t.Tensor | None = None

    @staticmethod
    def forward(ctx, mu, q, s, alpha, albedo, k_j, cam_rotation, cam_translation, fx, fy, cx,
                cy, height, width):
        if crc is None:
            raise ImportError(
                "custom_rasterizer_cuda is not available; build it with "
                "`python custom-3dgs-cuda_b200/build.py`"
            )
        num_gaussians = mu.shape[0]
        mu, q, s = mu.contiguous(), q.contiguous(), s.contiguous()
        alpha, albedo, k_j = alpha.contiguous(), albedo.contiguous(), k_j.contiguous()
        cam_rotation = cam_rotation.contiguous()
        cam_translation = cam_translation.contiguous()
        fx_f, fy_f, cx_f, cy_f = float(fx), float(fy), float(cx), float(cy)
        img_h, img_w = int(height), int(width)

        cam_position = (-t.matmul(cam_rotation.T, cam_translation)).reshape(3).contiguous()
        mean_2d, cov_2d, depths = crc.project(
            num_gaussians, mu, q, s, cam_rotation, cam_translation, fx_f, fy_f, cx_f, cy_f
        )
        RasterizeFunction.last_radii2d = _screen_radii(cov_2d)
        colors = crc.SH(num_gaussians, cam_position, mu, albedo, k_j)
        rendered_img, sorted_ids, tile_ranges, final_T, n_contrib = crc.rasterize(
            num_gaussians, depths, mean_2d, cov_2d, colors, alpha, img_h, img_w
        )
        ctx.save_for_backward(
            mean_2d, cov_2d, colors, alpha, sorted_ids, tile_ranges, final_T, n_contrib,
            mu, q, s, albedo, k_j, cam_rotation, cam_translation, cam_position,
        )
        ctx.num_gaussians = num_gaussians
        ctx.height, ctx.width = img_h, img_w
        ctx.fx, ctx.fy, ctx.cx, ctx.cy = fx_f, fy_f, cx_f, cy_f
        return rendered_img

    @staticmethod
    def backward(ctx, grad_output):
        (mean_2d, cov_2d, colors, alpha, sorted_ids, tile_ranges, final_T, n_contrib,
         mu, q, s, albedo, k_j, cam_rotation, cam_translation, cam_position) = ctx.saved_tensors
        mean_2d_grad, cov_2d_grad, colors_grad, alpha_grad = crc.backwards_rasterization(
            grad_output.contiguous(), mean_2d, cov_2d, colors, alpha, sorted_ids, tile_ranges,
            final_T, n_contrib, ctx.num_gaussians, ctx.height, ctx.width,
        )
        RasterizeFunction.last_mean2d_grad = mean_2d_grad.detach()
        albedo_grad, k_j_grad, mu_sh_grad = crc.backwards_SH(
            colors_grad, mu, albedo, k_j, cam_position
        )
        mu_grad, q_grad, s_grad = crc.backwards_projection(
            mean_2d_grad, cov_2d_grad, mu, q, s, cam_rotation, cam_translation,
            ctx.fx, ctx.fy, ctx.cx, ctx.cy,
        )
        mu_grad = mu_grad + mu_sh_grad
        alpha_grad = alpha_grad.view_as(alpha) if alpha_grad.numel() == alpha.numel() else alpha_grad
        return (mu_grad, q_grad, s_grad, alpha_grad, albedo_grad, k_j_grad,
                None, None, None, None, None, None, None, None)


def rasterize(gaussians: gaussian, image: dict) -> t.Tensor:
    """Renders `gaussians` from the camera in `image` (keys R, T, fx, fy, cx, cy, height,
    width); opacity logits go through a sigmoid first."""
    RasterizeFunction.last_mean2d_grad = None
    RasterizeFunction.last_radii2d = None
    return RasterizeFunction.apply(
        gaussians.mu, gaussians.q, gaussians.s, t.sigmoid(gaussians.alpha), gaussians.A,
        gaussians.k_j, image["R"], image["T"], image["fx"], image["fy"], image["cx"],
        image["cy"], image["height"], image["width"],
    )
