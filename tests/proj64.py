"""Float64 torch restatement of the reference's projection (csrc/forward/projection.cu:33-105)
for gradient checks: autograd through it gives the exact derivative of the forward that the
kernels implement. TEST INFRASTRUCTURE ONLY.

`project64(mu, q, s, R, t, fx, fy, cx, cy, transpose_rotation=False)` returns
(mean2d[N,2], cov2d[N,3], rotation[N,3,3]) with the reference's near-plane cull (z <= 0.2 gives
zeros) and its (a, b, c) = (Sigma2_00 + 0.3, Sigma2_01, Sigma2_11 + 0.3) packing. The quaternion
is (w, x, y, z) and is normalised first; the rotation is the standard unit-quaternion matrix.
"""

from __future__ import annotations

import torch


def quat_rotation64(q: torch.Tensor) -> torch.Tensor:
    """A zero quaternion maps to the identity, as in the reference (its derivative is
    undefined there)."""
    norm = q.norm(dim=1, keepdim=True)
    qn = q / torch.where(norm > 0, norm, torch.ones_like(norm))
    w, x, y, z = qn.unbind(1)
    return torch.stack([
        torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], 1),
        torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], 1),
        torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], 1)], 1)


def project64(mu, q, s, R, t, fx, fy, cx, cy, rotation=None):
    """`rotation` overrides R(q) (an [N,3,3] tensor) when given."""
    mu, q, s = (torch.as_tensor(v).double() for v in (mu, q, s))
    R, t = (torch.as_tensor(v, device=mu.device).double() for v in (R, t))
    pc = mu @ R.T + t
    z = pc[:, 2]
    valid = z > 0.2
    zs = torch.where(valid, z, torch.ones_like(z))
    mean = torch.stack([fx * pc[:, 0] / zs + cx, fy * pc[:, 1] / zs + cy], 1)
    Rq = quat_rotation64(q) if rotation is None else rotation
    M = Rq * torch.exp(s)[:, None, :]
    Sc = R @ (M @ M.transpose(1, 2)) @ R.T
    J = torch.zeros(mu.shape[0], 2, 3, dtype=torch.float64, device=mu.device)
    J[:, 0, 0] = fx / zs
    J[:, 0, 2] = -fx * pc[:, 0] / zs ** 2
    J[:, 1, 1] = fy / zs
    J[:, 1, 2] = -fy * pc[:, 1] / zs ** 2
    C2 = J @ Sc @ J.transpose(1, 2)
    cov = torch.stack([C2[:, 0, 0] + 0.3, C2[:, 0, 1], C2[:, 1, 1] + 0.3], 1)
    zero = torch.zeros((), dtype=torch.float64)
    return (torch.where(valid[:, None], mean, zero), torch.where(valid[:, None], cov, zero), Rq)


def projection_grads64(g_mean2d, g_cov2d, mu, q, s, R, t, fx, fy, cx, cy):
    """(d mu, d q, d s) of sum(g_mean2d * mean2d + g_cov2d * cov2d), exact in float64."""
    mu64, q64, s64 = (torch.as_tensor(v).double().clone().requires_grad_(True) for v in (mu, q, s))
    m, c, _ = project64(mu64, q64, s64, R, t, fx, fy, cx, cy)
    L = ((m * torch.as_tensor(g_mean2d, device=m.device).double()).sum()
         + (c * torch.as_tensor(g_cov2d, device=m.device).double()).sum())
    return torch.autograd.grad(L, (mu64, q64, s64))


def transposed_rotation_q_grad64(g_mean2d, g_cov2d, mu, q, s, R, t, fx, fy, cx, cy):
    """The quaternion gradient the reference's formula computes (csrc/backward/
    projection_backward.cu:116-138): with G = dL/dR for the rotation R(q) the forward uses, it
    returns d/dq of sum_ij G_ij R(q)_ji, i.e. the derivative of the TRANSPOSED rotation, then
    projects it through the normalisation like the true gradient."""
    q64 = torch.as_tensor(q).double().clone().requires_grad_(True)
    Rq = quat_rotation64(q64).detach().requires_grad_(True)
    m, c, _ = project64(mu, q64.detach(), s, R, t, fx, fy, cx, cy, rotation=Rq)
    L = ((m * torch.as_tensor(g_mean2d, device=m.device).double()).sum()
         + (c * torch.as_tensor(g_cov2d, device=m.device).double()).sum())
    (G,) = torch.autograd.grad(L, (Rq,))
    Lt = (G * quat_rotation64(q64).transpose(1, 2)).sum()
    (gq,) = torch.autograd.grad(Lt, (q64,))
    return gq
