"""The fused L1 + SSIM loss kernels against the reference's loss semantics.

The reference trainer's loss is `calculate_loss` (gaussian_splatting/utils/loss.py:15-33):
0.8 * mean|gt - img| + 0.2 * (1 - ssim(img, gt, data_range=1.0)), with torchmetrics'
structural_similarity_index_measure on NCHW images clamped to [0, 1] (loss.py:8-10).
torchmetrics is a dependency of the reference (requirements.txt: torchmetrics>=1.0, no version
pinned) that is not installed here, so `torchmetrics_ssim64` restates its published algorithm
(torchmetrics.functional.image.ssim, `_ssim_update` with gaussian_kernel=True, sigma=1.5,
k1=0.01, k2=0.03, reduction "elementwise_mean"):
  * window: kernel size int(3.5 * sigma + 0.5) * 2 + 1 = 11; 1-D taps exp(-(d / sigma)^2 / 2)
    for d = -5..5, normalised to sum 1; the 2-D window is their outer product, per channel;
  * both images reflect-padded by 5 on every side; depthwise convolution (no padding) of
    x, y, x*x, y*y, x*y;
  * var_x = E[x^2] - mu_x^2 and var_y clamped at 0; cov = E[xy] - mu_x mu_y;
  * SSIM map ((2 mu_x mu_y + C1)(2 cov + C2)) / ((mu_x^2 + mu_y^2 + C1)(var_x + var_y + C2)),
    C1 = (0.01 * data_range)^2, C2 = (0.03 * data_range)^2;
  * the map cropped by 5 on every side and averaged.
It runs in float64 here. The kernels must give the loss within 1e-5 relative and the gradient
within 1e-4 relative (floor 1e-4 x RMS).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def torchmetrics_ssim64(preds_hwc: torch.Tensor, target_hwc: torch.Tensor) -> torch.Tensor:
    x = preds_hwc.double().permute(2, 0, 1).unsqueeze(0).clamp(0.0, 1.0)
    y = target_hwc.double().permute(2, 0, 1).unsqueeze(0).clamp(0.0, 1.0)
    sigma, data_range = 1.5, 1.0
    ks = int(3.5 * sigma + 0.5) * 2 + 1
    pad = (ks - 1) // 2
    d = torch.arange((1 - ks) / 2, (1 + ks) / 2, 1, dtype=torch.float64, device=x.device)
    g = torch.exp(-torch.pow(d / sigma, 2) / 2)
    g = (g / g.sum()).unsqueeze(0)
    kernel = torch.matmul(g.t(), g).expand(3, 1, ks, ks)
    xp = F.pad(x, (pad, pad, pad, pad), mode="reflect")
    yp = F.pad(y, (pad, pad, pad, pad), mode="reflect")
    out = F.conv2d(torch.cat((xp, yp, xp * xp, yp * yp, xp * yp)), kernel, groups=3)
    mu_x, mu_y, exx, eyy, exy = out.split(1)
    var_x = torch.clamp(exx - mu_x.pow(2), min=0.0)
    var_y = torch.clamp(eyy - mu_y.pow(2), min=0.0)
    cov = exy - mu_x * mu_y
    c1, c2 = (0.01 * data_range) ** 2, (0.03 * data_range) ** 2
    full = ((2 * mu_x * mu_y + c1) * (2 * cov + c2)) / (
        (mu_x.pow(2) + mu_y.pow(2) + c1) * (var_x + var_y + c2))
    return full[..., pad:-pad, pad:-pad].reshape(1, -1).mean(-1)[0]


def reference_loss64(img_hwc: torch.Tensor, gt_hwc: torch.Tensor) -> torch.Tensor:
    l1 = torch.mean(torch.abs(gt_hwc.double() - img_hwc.double()))
    return 0.8 * l1 + 0.2 * (1.0 - torchmetrics_ssim64(img_hwc, gt_hwc))


def _pair(H, W, seed, spill=False):
    g = torch.Generator("cpu").manual_seed(seed)
    target = torch.rand(H, W, 3, generator=g)
    img = target + 0.2 * torch.randn(H, W, 3, generator=g)
    if not spill:
        img = img.clamp(0, 1)
    return img, target


@pytest.mark.parametrize("shape", [(64, 96), (1080, 1920), (37, 53), (11, 200)])
@pytest.mark.parametrize("spill", [False, True], ids=["in_range", "outside_0_1"])
def test_fused_l1_ssim_matches_torchmetrics_semantics(cuda_device, shape, spill):
    from gs3d_b200.loss import l1_ssim_loss

    H, W = shape
    img, target = _pair(H, W, H * 7 + W, spill)
    x = img.to(cuda_device).requires_grad_(True)
    loss = l1_ssim_loss(x, target.to(cuda_device))
    loss.backward()
    x64 = img.double().to(cuda_device).requires_grad_(True)
    ref = reference_loss64(x64, target.double().to(cuda_device))
    ref.backward()
    assert abs(float(loss) - float(ref)) <= 1e-5 * abs(float(ref))
    a = x.grad.double().cpu().numpy()
    b = x64.grad.cpu().numpy()
    rms = float(np.sqrt(np.mean(b * b)))
    np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-4 * rms)


def test_fused_loss_matches_the_torch_formulation(cuda_device):
    """train_step.reconstruction_loss (valid convolution) is the same function."""
    from gs3d_b200.loss import l1_ssim_loss
    from gs3d_b200.train_step import gaussian_window, reconstruction_loss

    img, target = _pair(90, 70, 5, spill=True)
    x = img.double().to(cuda_device)
    ref = reference_loss64(x, target.double().to(cuda_device))
    mine = reconstruction_loss(x, target.double().to(cuda_device),
                               gaussian_window(device=cuda_device, dtype=torch.float64))
    assert abs(float(mine) - float(ref)) <= 1e-12
    fused = l1_ssim_loss(img.to(cuda_device), target.to(cuda_device))
    assert abs(float(fused) - float(ref)) <= 1e-5 * abs(float(ref))


def test_fused_l1_ssim_is_deterministic(cuda_device):
    from gs3d_b200.loss import l1_ssim_loss

    g = torch.Generator("cpu").manual_seed(3)
    a = torch.rand(270, 480, 3, generator=g).to(cuda_device)
    b = torch.rand(270, 480, 3, generator=g).to(cuda_device)
    assert float(l1_ssim_loss(a, b)) == float(l1_ssim_loss(a, b))


def test_fused_l1_ssim_rejects_images_below_the_window(cuda_device):
    from gs3d_b200.loss import l1_ssim_loss

    a = torch.rand(10, 64, 3, device=cuda_device)
    with pytest.raises(RuntimeError, match="at least 11 x 11"):
        l1_ssim_loss(a, a.clone())


@pytest.mark.parametrize("shape", [(1080, 1920), (37, 53)])
def test_ssim_backward_tile_copies_match_warp_loads(cuda_device, shape, monkeypatch):
    """The SSIM backward reads its derivative-map planes through tile copies of the tensor
    memory accelerator; its fallback (the warps' own loads, for a driver without the
    tensor-map entry point) must give the same bits."""
    from gs3d_b200.loss import l1_ssim_value_and_grad

    H, W = shape
    img, target = _pair(H, W, 31 + H, spill=True)
    x, y = img.to(cuda_device), target.to(cuda_device)
    loss_a, grad_a = l1_ssim_value_and_grad(x, y, 0.2)
    monkeypatch.setenv("GS3D_SSIM_NO_TMA", "1")
    loss_b, grad_b = l1_ssim_value_and_grad(x, y, 0.2)
    assert torch.equal(loss_a, loss_b) and torch.equal(grad_a, grad_b)
