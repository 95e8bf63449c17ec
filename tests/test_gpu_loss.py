"""The fused L1 + SSIM loss kernels against the torch formulation of the same loss
(train_step.reconstruction_loss: 11x11 Gaussian window, sigma 1.5, zero padding) evaluated in
float64: loss within 1e-5 relative, gradient within 1e-4 relative (floor 1e-4 x RMS)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(64, 96), (1080, 1920), (37, 53), (11, 200)])
def test_fused_l1_ssim_matches_torch(cuda_device, shape):
    from gs3d_b200.loss import l1_ssim_loss
    from gs3d_b200.train_step import gaussian_window, reconstruction_loss

    H, W = shape
    g = torch.Generator("cpu").manual_seed(H * 7 + W)
    target = torch.rand(H, W, 3, generator=g)
    img = (target + 0.2 * torch.randn(H, W, 3, generator=g)).clamp(0, 1)
    x = img.to(cuda_device).requires_grad_(True)
    loss = l1_ssim_loss(x, target.to(cuda_device))
    loss.backward()
    x64 = img.double().to(cuda_device).requires_grad_(True)
    ref = reconstruction_loss(x64, target.double().to(cuda_device),
                              gaussian_window(device=cuda_device).double())
    ref.backward()
    assert abs(float(loss) - float(ref)) <= 1e-5 * abs(float(ref))
    a = x.grad.double().cpu().numpy()
    b = x64.grad.cpu().numpy()
    rms = float(np.sqrt(np.mean(b * b)))
    np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-4 * rms)


def test_fused_l1_ssim_is_deterministic(cuda_device):
    from gs3d_b200.loss import l1_ssim_loss

    g = torch.Generator("cpu").manual_seed(3)
    a = torch.rand(270, 480, 3, generator=g).to(cuda_device)
    b = torch.rand(270, 480, 3, generator=g).to(cuda_device)
    assert float(l1_ssim_loss(a, b)) == float(l1_ssim_loss(a, b))
