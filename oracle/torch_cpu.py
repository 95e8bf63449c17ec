"""PyTorch-on-CPU restatement of the rasterizer's forward, differentiated by autograd.

Test and benchmark infrastructure, not product code: bench.py times it on the host cores
(the scene meant for a PyTorch CPU evaluation) and tests/test_oracle_torch.py
checks it against the C oracle (oracle/gs_oracle.c). It follows the reference's math:
  * projection: csrc/forward/projection.cu:28-105 (cull z <= 0.2 to zeros; a, c += 0.3);
  * SH colour: csrc/forward/SH.cu:57-93 (direction without epsilon, clamp to [0, 1]);
  * binning: csrc/forward/rasterize.cu:19-59 (radius and tile rectangle) and :79-135 (keys
    tile << 32 | depth bits), the stable 64-bit sort of :416-435 and the ranges of :146-165;
  * blend: csrc/forward/rasterize.cu:188-280 (skip power > 0 or alpha < 1/255, alpha capped at
    0.99, stop after the Gaussian that takes T below 1e-4).
Each tile is evaluated densely (its 256 pixels against its whole list): transmittance by
cumulative products, the stop rule as a mask. The masks carry no gradient, as in the
reference's backward. Floats are rounded as torch rounds them (no fused multiply-adds), so
agreement with the kernels is to tolerance, not bit for bit.
"""

from __future__ import annotations

import torch

TILE = 16
_C0 = 0.28209479177387814
_C1 = 0.4886025119029199
_C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792,
       0.5462742152960396)
_C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
       -0.4570457994644658, 1.445305721320277, -0.5900435899266435)


def quat_rotation(q: torch.Tensor) -> torch.Tensor:
    """[N, 3, 3] rotation of the normalised quaternion (w, x, y, z)."""
    q = q * torch.rsqrt((q * q).sum(1, keepdim=True))
    w, x, y, z = q.unbind(1)
    return torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], 1).reshape(-1, 3, 3)


def project(mu, q, s, R, t, fx, fy, cx, cy):
    """(mean2d [N, 2], cov2d [N, 3], depths [N]); culled Gaussians get zeros."""
    pc = mu @ R.T + t
    x, y, z = pc.unbind(1)
    keep = z > 0.2
    zs = torch.where(keep, z, torch.ones_like(z))
    mean2d = torch.stack([fx * x / zs + cx, fy * y / zs + cy], 1)
    M = quat_rotation(q) * torch.exp(s)[:, None, :]
    sigma_c = R @ (M @ M.transpose(1, 2)) @ R.T
    J = torch.zeros(mu.shape[0], 2, 3, dtype=mu.dtype)
    J[:, 0, 0] = fx / zs
    J[:, 0, 2] = -fx * x / (zs * zs)
    J[:, 1, 1] = fy / zs
    J[:, 1, 2] = -fy * y / (zs * zs)
    cov = J @ sigma_c @ J.transpose(1, 2)
    cov2d = torch.stack([cov[:, 0, 0] + 0.3, cov[:, 0, 1], cov[:, 1, 1] + 0.3], 1)
    k = keep[:, None].to(mu.dtype)
    return mean2d * k, cov2d * k, z * keep.to(mu.dtype)


def sh_colour(cam, mu, A, kj):
    """[N, 3] colour, degrees 0..3, clamped to [0, 1]."""
    v = mu - cam
    d = v / torch.sqrt((v * v).sum(1, keepdim=True))
    x, y, z = d.unbind(1)
    xx, yy, zz = x * x, y * y, z * z
    Y = torch.stack([
        -_C1 * y, _C1 * z, -_C1 * x,
        _C2[0] * x * y, _C2[1] * y * z, _C2[2] * (2 * zz - xx - yy), _C2[3] * x * z,
        _C2[4] * (xx - yy),
        _C3[0] * y * (3 * xx - yy), _C3[1] * x * y * z, _C3[2] * y * (4 * zz - xx - yy),
        _C3[3] * z * (2 * zz - 3 * xx - 3 * yy), _C3[4] * x * (4 * zz - xx - yy),
        _C3[5] * z * (xx - yy), _C3[6] * x * (xx - 3 * yy)], 1)
    rgb = 0.5 + _C0 * A + (Y[:, :, None] * kj).sum(1)
    return rgb.clamp(0.0, 1.0)


def tile_lists(mean2d, cov2d, depths, H, W):
    """(sorted Gaussian ids, ranges [T, 2]) of the reference's binning and stable sort."""
    with torch.no_grad():
        tx, ty = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
        a, b, c = cov2d.unbind(1)
        det = a * c - b * b
        mid = 0.5 * (a + c)
        lam = mid + torch.sqrt(torch.clamp(mid * mid - det, min=0.1))
        r = torch.ceil(3.0 * torch.sqrt(lam))
        mx, my = mean2d.unbind(1)
        x0 = torch.clamp(torch.floor(mx - r), min=0).long() // TILE
        x1 = (torch.clamp(torch.ceil(mx + r), max=W).long() + TILE - 1) // TILE
        y0 = torch.clamp(torch.floor(my - r), min=0).long() // TILE
        y1 = (torch.clamp(torch.ceil(my + r), max=H).long() + TILE - 1) // TILE
        x0, x1 = x0.clamp(0, tx), x1.clamp(0, tx)
        y0, y1 = y0.clamp(0, ty), y1.clamp(0, ty)
        ok = det > 0
        w = torch.where(ok, (x1 - x0).clamp(min=0), torch.zeros_like(x0))
        h = torch.where(ok, (y1 - y0).clamp(min=0), torch.zeros_like(y0))
        counts = w * h
        gid = torch.repeat_interleave(torch.arange(mean2d.shape[0]), counts)
        local = torch.arange(int(counts.sum())) - torch.repeat_interleave(
            torch.cumsum(counts, 0) - counts, counts)
        tile = ((y0[gid] + local // w[gid]) * tx + x0[gid] + local % w[gid])
        dbits = depths.detach().contiguous().view(torch.int32).long() & 0xFFFFFFFF
        keys = (tile << 32) | dbits[gid]
        order = torch.sort(keys, stable=True).indices
        sorted_tiles = tile[order]
        T = tx * ty
        bounds = torch.searchsorted(sorted_tiles, torch.arange(T + 1))
        ranges = torch.stack([bounds[:-1], bounds[1:]], 1)
        return gid[order], ranges


def blend(mean2d, cov2d, colours, opacity, ids, ranges, H, W):
    """(image [H, W, 3], final_T [H, W]) of the front-to-back blend."""
    tx = (W + TILE - 1) // TILE
    img = torch.zeros(H, W, 3, dtype=mean2d.dtype)
    final_T = torch.ones(H, W, dtype=mean2d.dtype)
    a, b, c = cov2d.unbind(1)
    det = a * c - b * b
    inv = torch.where(det > 0, 1.0 / torch.where(det > 0, det, torch.ones_like(det)),
                      torch.zeros_like(det))
    conic = torch.stack([c * inv, -b * inv, a * inv], 1)
    for tile, (start, end) in enumerate(ranges.tolist()):
        if end <= start:
            continue
        px0, py0 = (tile % tx) * TILE, (tile // tx) * TILE
        xs = torch.arange(px0, min(px0 + TILE, W), dtype=mean2d.dtype)
        ys = torch.arange(py0, min(py0 + TILE, H), dtype=mean2d.dtype)
        py, px = torch.meshgrid(ys, xs, indexing="ij")
        g = ids[start:end]
        dx = px.reshape(-1, 1) - mean2d[g, 0]
        dy = py.reshape(-1, 1) - mean2d[g, 1]
        q = conic[g]
        power = -0.5 * (q[:, 0] * dx * dx + 2.0 * q[:, 1] * dx * dy + q[:, 2] * dy * dy)
        alpha = torch.clamp(opacity[g] * torch.exp(power), max=0.99)
        valid = (power <= 0) & (alpha >= 1.0 / 255.0)
        a_eff = torch.where(valid, alpha, torch.zeros_like(alpha))
        trans = torch.cumprod(1.0 - a_eff, 1)
        before = torch.cat([torch.ones_like(trans[:, :1]), trans[:, :-1]], 1)
        applied = valid & (before.detach() >= 1e-4)  # after the stop nothing applies
        w_eff = torch.where(applied, a_eff * before, torch.zeros_like(a_eff))
        rows, cols = ys.long(), xs.long()
        img[rows[0]:rows[-1] + 1, cols[0]:cols[-1] + 1] = (w_eff @ colours[g]).reshape(
            len(rows), len(cols), 3)
        keep = torch.where(applied, 1.0 - a_eff, torch.ones_like(a_eff))
        final_T[rows[0]:rows[-1] + 1, cols[0]:cols[-1] + 1] = torch.prod(keep, 1).reshape(
            len(rows), len(cols))
    return img, final_T


def render(mu, q, s, alpha_logit, A, kj, R, t, fx, fy, cx, cy, H, W):
    """(image, final_T) of the reference wrapper's forward from the raw parameters."""
    mean2d, cov2d, depths = project(mu, q, s, R, t, fx, fy, cx, cy)
    cam = -(R.T @ t)
    colours = sh_colour(cam, mu, A, kj)
    opacity = torch.sigmoid(alpha_logit).reshape(-1)
    ids, ranges = tile_lists(mean2d, cov2d, depths, H, W)
    return blend(mean2d, cov2d, colours, opacity, ids, ranges, H, W)


def step_seconds(scene, view, target, reps: int = 3) -> tuple[float, int]:
    """Median seconds of one forward + L1 backward (BASELINE config 0's step) on the host
    cores, and the thread count used."""
    import time

    threads = torch.get_num_threads()
    params = [p.detach().clone().requires_grad_(True) for p in scene.params()]
    R, t = view.R.float(), view.T.float()
    times = []
    for _ in range(reps):
        for p in params:
            p.grad = None
        t0 = time.perf_counter()
        img, _ = render(*params, R, t, view.fx, view.fy, view.cx, view.cy, view.height,
                        view.width)
        (img - target).abs().mean().backward()
        times.append(time.perf_counter() - t0)
    times.sort()
    return times[len(times) // 2], threads
