"""The PyTorch CPU restatement (oracle/torch_cpu.py, timed by bench.py on BASELINE config 0)
against the C oracle on config 0: the same forward to float tolerance, and its autograd
gradients against the oracle's analytic backward chain (blend, SH, projection backward) for the
means, log-scales, opacity and SH coefficients. The quaternion is left out: the reference's
quaternion gradient, which the oracle restates, is the derivative of the transposed rotation
(tests/test_oracle_kat.py), autograd's that of the forward."""

from __future__ import annotations

import numpy as np
import torch

from gs3d_b200 import scenes
from oracle import oracle as O
from oracle import torch_cpu as TC


def _close(a, b, what, rtol, outlier_frac):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64).reshape(a.shape)
    rms = float(np.sqrt(np.mean(b * b))) or 1.0
    err = np.abs(a - b)
    out = int((err > rtol * (np.abs(b) + rms)).sum())
    assert out <= outlier_frac * b.size, f"{what}: {out}/{b.size} beyond {rtol}, worst {err.max():.3e}"


def test_torch_restatement_matches_c_oracle_on_config0():
    O.build()
    sc = scenes.config0(0)
    view = sc.views[0]
    R, t = view.R.float(), view.T.float()
    H, W = view.height, view.width
    target = torch.rand(H, W, 3, generator=torch.Generator().manual_seed(1))
    params = [p.detach().clone().requires_grad_(True) for p in sc.params()]
    mu, q, s, al, A, kj = params
    img, final_T = TC.render(mu, q, s, al, A, kj, R, t, view.fx, view.fy, view.cx, view.cy, H, W)
    loss = (img - target).abs().mean()
    loss.backward()

    op = torch.sigmoid(sc.alpha).numpy().reshape(-1)
    Rn, tn = R.numpy(), t.numpy()
    out = O.render(sc.mu.numpy(), sc.q.numpy(), sc.s.numpy(), op, sc.A.numpy(), sc.k_j.numpy(),
                   Rn, tn, view.fx, view.fy, view.cx, view.cy, H, W)
    _close(img.detach().numpy(), out["img"], "image", 1e-4, 1e-3)
    _close(final_T.detach().numpy(), out["final_T"], "final_T", 1e-4, 1e-3)

    gimg = (np.sign(out["img"] - target.numpy()) / out["img"].size).astype(np.float32)
    gm, gc, gcol, ga, _ = O.rasterize_backward(gimg, out["mean2d"], out["cov2d"], out["colors"],
                                               op, out["sorted_ids"], out["tile_ranges"],
                                               out["final_T"], out["n_contrib"], H, W)
    gA, gkj, gmu_sh = O.sh_backward(gcol, sc.mu.numpy(), sc.A.numpy(), sc.k_j.numpy(),
                                    O.camera_position(Rn, tn))
    gmu, _gq, gs = O.project_backward(gm, gc, sc.mu.numpy(), sc.q.numpy(), sc.s.numpy(), Rn, tn,
                                      view.fx, view.fy, view.cx, view.cy)
    g_logit = np.asarray(ga).reshape(-1) * op * (1.0 - op)
    _close(mu.grad.numpy(), np.asarray(gmu) + np.asarray(gmu_sh), "mu", 1e-3, 1e-2)
    _close(s.grad.numpy(), gs, "log-scales", 1e-3, 1e-2)
    _close(al.grad.numpy().reshape(-1), g_logit, "opacity logits", 1e-3, 1e-2)
    _close(A.grad.numpy(), gA, "SH DC", 1e-3, 1e-2)
    _close(kj.grad.numpy(), gkj, "SH rest", 1e-3, 1e-2)
