"""The torch formulation of the training-step loss (train_step.reconstruction_loss, used by the
CPU process-group tests) equals the float64 restatement of torchmetrics' SSIM algorithm that
the GPU loss tests check the fused kernels against (reflect padding then the 5-pixel crop)."""

from __future__ import annotations

import torch

from tests.test_gpu_loss import reference_loss64, torchmetrics_ssim64


def test_torch_formulation_matches_torchmetrics_restatement():
    from gs3d_b200.train_step import gaussian_window, reconstruction_loss, ssim

    g = torch.Generator("cpu").manual_seed(11)
    for H, W in ((11, 11), (23, 40), (64, 33)):
        t = torch.rand(H, W, 3, generator=g, dtype=torch.float64)
        x = t + 0.3 * torch.randn(H, W, 3, generator=g, dtype=torch.float64)  # spills out of [0, 1]
        win = gaussian_window(dtype=torch.float64)
        assert abs(float(ssim(x, t, win)) - float(torchmetrics_ssim64(x, t))) < 1e-12
        assert abs(float(reconstruction_loss(x, t, win)) - float(reference_loss64(x, t))) < 1e-12


def test_identical_images_have_ssim_one():
    g = torch.Generator("cpu").manual_seed(12)
    x = torch.rand(30, 30, 3, generator=g, dtype=torch.float64)
    assert abs(float(torchmetrics_ssim64(x, x)) - 1.0) < 1e-12
