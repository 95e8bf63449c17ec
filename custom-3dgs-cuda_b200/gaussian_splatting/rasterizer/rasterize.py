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


class RasterizeFunction(t.autograd.Function):
    """Projection -> SH colour -> tile binning/sort -> alpha blend, and the reverse.

    Runs the fused render path (custom_rasterizer_cuda.render: two C-ABI calls per direction
    instead of the reference's six ops); its outputs equal chaining the six ops. It bins each
    splat only into the tiles where it can pass the opacity test (GS_RENDER_TIGHT_BINS): the
    pairs it drops fail that test at every pixel of their tile, so the image, transmittance,
    radii and gradients are those of the reference's binning, from shorter tile lists (the
    lists themselves are not outputs of this function).
    """

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
        from custom_rasterizer_cuda.render import render_forward

        mu, q, s = mu.contiguous(), q.contiguous(), s.contiguous()
        alpha, albedo, k_j = alpha.contiguous(), albedo.contiguous(), k_j.contiguous()
        cam_rotation = cam_rotation.contiguous()
        cam_translation = cam_translation.contiguous()
        for tensor, name in ((mu, "mu"), (q, "q"), (s, "s"), (alpha, "alpha"), (albedo, "albedo"),
                             (k_j, "k_j"), (cam_rotation, "cam_rotation"),
                             (cam_translation, "cam_translation")):
            if not tensor.is_cuda or tensor.dtype != t.float32:
                raise RuntimeError(f"{name} must be a CUDA FP32 tensor")
        n = mu.shape[0]
        if q.numel() < 4 * n or s.numel() < 3 * n or alpha.numel() != n or \
                albedo.numel() < 3 * n or k_j.numel() < 45 * n:
            raise RuntimeError("Gaussian parameters must hold N rows")
        fx_f, fy_f, cx_f, cy_f = float(fx), float(fy), float(cx), float(cy)
        img_h, img_w = int(height), int(width)

        cam_position = (-t.matmul(cam_rotation.T, cam_translation)).reshape(3).contiguous()
        img, radii, state = render_forward(mu, q, s, alpha, albedo, k_j, cam_rotation,
                                           cam_translation, cam_position, fx_f, fy_f, cx_f, cy_f,
                                           img_h, img_w, tight_bins=True)
        RasterizeFunction.last_radii2d = radii
        ctx.save_for_backward(mu, q, s, alpha, albedo, k_j, cam_rotation, cam_translation,
                              cam_position)
        ctx.state = state
        ctx.fx, ctx.fy, ctx.cx, ctx.cy = fx_f, fy_f, cx_f, cy_f
        return img

    @staticmethod
    def backward(ctx, grad_output):
        from custom_rasterizer_cuda.render import render_backward

        (mu, q, s, alpha, albedo, k_j, cam_rotation, cam_translation,
         cam_position) = ctx.saved_tensors
        g_mu, g_q, g_s, g_alpha, g_albedo, g_kj, g_mean2d = render_backward(
            ctx.state, grad_output, mu, q, s, albedo, k_j, cam_rotation, cam_translation,
            cam_position, ctx.fx, ctx.fy, ctx.cx, ctx.cy)
        RasterizeFunction.last_mean2d_grad = g_mean2d
        return (g_mu, g_q, g_s, g_alpha.view_as(alpha), g_albedo, g_kj,
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
