"""The training step's photometric loss, 0.8 * L1 + 0.2 * (1 - SSIM), as one autograd op over
the fused kernels of libgs3d_b200 (gs_l1_ssim_forward / gs_l1_ssim_backward).

`l1_ssim_loss(img, target)` matches the reference's `calculate_loss`
(gaussian_splatting/utils/loss.py:15-33: torchmetrics SSIM with data_range 1.0 on the images
clamped to [0, 1], 11x11 Gaussian window, sigma 1.5, mean over the interior positions) and
`train_step.reconstruction_loss` (its torch formulation) on [H, W, 3] fp32 CUDA images of at
least 11 x 11 pixels.
"""

from __future__ import annotations

import torch

from custom_rasterizer_cuda import _lib

LAMBDA_DSSIM = 0.2


class FusedL1SSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img: torch.Tensor, target: torch.Tensor, lambda_dssim: float = LAMBDA_DSSIM):
        if not (img.is_cuda and target.is_cuda):
            raise RuntimeError("l1_ssim_loss needs CUDA tensors")
        if img.dim() != 3 or img.shape[2] != 3 or img.shape != target.shape:
            raise RuntimeError("l1_ssim_loss expects two [H, W, 3] images of the same shape")
        img = img.contiguous().float()
        target = target.contiguous().float()
        H, W = int(img.shape[0]), int(img.shape[1])
        dev = img.device
        ws_bytes = _lib.lib.gs_l1_ssim_workspace_size(H, W)
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
        loss = torch.empty((), device=dev, dtype=torch.float32)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib.gs_l1_ssim_forward(
                H, W, img.data_ptr(), target.data_ptr(), float(lambda_dssim), ws.data_ptr(),
                ws_bytes, loss.data_ptr(), None, torch.cuda.current_stream(dev).cuda_stream))
        ctx.save_for_backward(img, target, ws)
        ctx.lambda_dssim = float(lambda_dssim)
        return loss

    @staticmethod
    def backward(ctx, grad_loss: torch.Tensor):
        img, target, ws = ctx.saved_tensors
        H, W = int(img.shape[0]), int(img.shape[1])
        dev = img.device
        grad_loss = grad_loss.contiguous().float().reshape(())
        grad = torch.empty_like(img)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib.gs_l1_ssim_backward(
                H, W, img.data_ptr(), target.data_ptr(), ctx.lambda_dssim, ws.data_ptr(),
                ws.numel(), grad_loss.data_ptr(), grad.data_ptr(),
                torch.cuda.current_stream(dev).cuda_stream))
        return grad, None, None


def l1_ssim_loss(img: torch.Tensor, target: torch.Tensor,
                 lambda_dssim: float = LAMBDA_DSSIM) -> torch.Tensor:
    return FusedL1SSIM.apply(img, target, lambda_dssim)


class _OneCache:
    """A device scalar 1.0 per device (the upstream gradient of a loss used directly)."""

    def __init__(self) -> None:
        self._ones: dict = {}

    def get(self, dev) -> torch.Tensor:
        t = self._ones.get(dev)
        if t is None:
            t = self._ones[dev] = torch.ones((), device=dev, dtype=torch.float32)
        return t


_one = _OneCache()


def l1_ssim_value_and_grad(img: torch.Tensor, target: torch.Tensor,
                           lambda_dssim: float = LAMBDA_DSSIM,
                           grad_out: torch.Tensor | None = None):
    """(loss, dloss/dimg) in two kernel launches, outside autograd; [H, W, 3] fp32 CUDA."""
    img = img.contiguous()
    target = target.contiguous()
    H, W = int(img.shape[0]), int(img.shape[1])
    dev = img.device
    ws_bytes = _lib.lib.gs_l1_ssim_workspace_size(H, W)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    loss = torch.empty((), device=dev, dtype=torch.float32)
    grad = torch.empty_like(img) if grad_out is None else grad_out
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.gs_l1_ssim_forward(H, W, img.data_ptr(), target.data_ptr(),
                                               float(lambda_dssim), ws.data_ptr(), ws_bytes,
                                               loss.data_ptr(), None, stream))
        _lib.check(_lib.lib.gs_l1_ssim_backward(H, W, img.data_ptr(), target.data_ptr(),
                                                float(lambda_dssim), ws.data_ptr(), ws_bytes,
                                                _one.get(dev).data_ptr(), grad.data_ptr(),
                                                stream))
    return loss, grad
