"""Adaptive density control with the reference's API (gaussian_splatting/utils/adc.py of the
reference): the densification-statistic helpers and `adaptive_density_control(gaussians,
optimizer, ...) -> (gaussians, optimizer, stats)`.

The clone / split / prune / opacity-reset decisions and the compaction of the parameters and
the Adam moments run on the GPU in two library calls (gs_adc_plan, gs_adc_apply) instead of
the reference's chain of torch ops and host synchronisations; one host read of five totals
sizes the new tensors. The results equal the reference's, in the same order. The split offsets
are `z * std` with unit normals `z` from torch's global generator (the reference calls
`torch.normal(0, std)`: the same distribution, not the same draws) or given by the caller. The
rare case where every Gaussian would be pruned keeps the 10% most opaque through torch ops, as
the reference does.

The optimizer is the reference's torch Adam with its six named groups (`setup_optimizer` in
gaussian_splatting/utils/optim.py of the reference); each group's parameter is replaced by a
new Parameter and its `exp_avg` / `exp_avg_sq` by the compacted moments ("step" is kept).
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

import torch as t
from torch.nn import Parameter

from gaussian_splatting.scene.gaussian import gaussian

# The reference optimizer's group names (its setup_optimizer) and the Gaussian attribute each
# one holds: the names are the optimizer's interface, so they are kept.
_GROUPS = (("mu", "mu"), ("q", "q"), ("Scale", "s"), ("Opacity", "alpha"),
           ("Albedo Coefficient", "A"), ("Illumination Coefficients", "k_j"))
_GROUP_TO_ATTR = dict(_GROUPS)
_ORDER = tuple(attr for _, attr in _GROUPS)

# densification buffers and the trailing shape of each
_STATE_BUFFERS = (("xyz_grad_accum", (1,)), ("denom", (1,)), ("max_radii2D", ()))


def scene_extent_from_means(mu: t.Tensor) -> float:
    """Length of the diagonal of the means' bounding box (at least 1e-3)."""
    lo, hi = t.aminmax(mu, dim=0)
    return max(float(t.linalg.vector_norm(hi - lo)), 1e-3)


def scene_extent_from_cameras(cameras) -> float:
    """1.1 x the largest distance of a camera centre (-R^T t) from the centres' mean (at
    least 1e-3)."""
    centres = -t.einsum("nji,nj->ni", cameras.R, cameras.t)
    spread = t.linalg.vector_norm(centres - centres.mean(dim=0, keepdim=True), dim=1)
    return max(1.1 * float(spread.max()), 1e-3)


def ensure_densification_state(gaussians: gaussian) -> None:
    """Densification buffers (xyz_grad_accum [N,1], denom [N,1], max_radii2D [N]) allocated or
    resized to the current N: rows that survive keep their values, new rows start at zero."""
    n = int(gaussians.mu.shape[0])
    for name, tail in _STATE_BUFFERS:
        cur = getattr(gaussians, name, None)
        if cur is None or int(cur.shape[0]) != n:
            fresh = gaussians.mu.new_zeros((n, *tail))
            if cur is not None:
                keep = min(int(cur.shape[0]), n)
                fresh[:keep] = cur[:keep].reshape(keep, *tail)
            cur = fresh
        setattr(gaussians, name, cur.reshape(n, *tail))


def accumulate_densification_stats(gaussians: gaussian, mean2d_grad: t.Tensor | None = None, *,
                                   width: int | None = None, height: int | None = None) -> None:
    """Adds one view's screen-space gradient norms |dL/dmean2d * (W/2, H/2)| to xyz_grad_accum
    and counts them in denom, for Gaussians with a non-zero norm (the scale is 1 when the image
    size is not given). One library launch (gs_densify_stats) on the gradient's device."""
    if mean2d_grad is None or mean2d_grad.shape[0] != gaussians.mu.shape[0]:
        return
    ensure_densification_state(gaussians)
    if not mean2d_grad.is_cuda:
        raise RuntimeError("accumulate_densification_stats needs CUDA tensors")
    grad = mean2d_grad.detach().float()
    if grad.stride(-1) != 1 or grad.dim() != 2:
        grad = grad.reshape(grad.shape[0], -1).contiguous()
    sized = bool(width and height and width > 0 and height > 0)
    sx, sy = (width / 2.0, height / 2.0) if sized else (1.0, 1.0)
    from custom_rasterizer_cuda import _lib

    n = int(grad.shape[0])
    acc, den = gaussians.xyz_grad_accum, gaussians.denom
    if not (acc.is_contiguous() and den.is_contiguous()):
        raise RuntimeError("the densification buffers must be contiguous")
    with t.cuda.device(grad.device):
        _lib.check(_lib.lib.gs_densify_stats(
            n, grad.data_ptr(), grad.stride(0), float(sx), float(sy), acc.data_ptr(),
            den.data_ptr(), None, t.cuda.current_stream(grad.device).cuda_stream))


def update_max_radii2d(gaussians: gaussian, radii: t.Tensor | None) -> None:
    """Running per-Gaussian maximum of the screen radius."""
    if radii is None or radii.shape[0] != gaussians.mu.shape[0]:
        return
    ensure_densification_state(gaussians)
    gaussians.max_radii2D = radii.detach().maximum(gaussians.max_radii2D)


def clamp_log_scales(gaussians: gaussian, scene_extent: float) -> None:
    """Caps every log-scale at log(0.1 x the scene extent) (floor 1e-7 before the log)."""
    cap = math.log(max(scene_extent * 0.1, 1e-7))
    gaussians.s.data.clamp_(max=cap)


def _group_state(optimizer, name):
    group = next(g for g in optimizer.param_groups if _GROUP_TO_ATTR[g["name"]] == name)
    old = group["params"][0]
    return group, old, optimizer.state.get(old, None)


def _replace(optimizer, name, new_param, exp_avg, exp_avg_sq):
    group, old, stored = _group_state(optimizer, name)
    group["params"][0] = new_param
    if stored is None:
        return
    new_state: dict[str, Any] = {}
    for key, value in stored.items():
        if key == "exp_avg" and exp_avg is not None:
            new_state[key] = exp_avg
        elif key == "exp_avg_sq" and exp_avg_sq is not None:
            new_state[key] = exp_avg_sq
        else:
            new_state[key] = value
    del optimizer.state[old]
    optimizer.state[new_param] = new_state


def _reset_stats(gaussians: gaussian) -> None:
    n = gaussians.mu.shape[0]
    kw = dict(device=gaussians.mu.device, dtype=gaussians.mu.dtype)
    gaussians.xyz_grad_accum = t.zeros(n, 1, **kw)
    gaussians.denom = t.zeros(n, 1, **kw)
    gaussians.max_radii2D = t.zeros(n, **kw)


def adaptive_density_control(gaussians: gaussian, optimizer: t.optim.Optimizer, *,
                             grad_threshold: float = 0.00005, percent_dense: float = 0.01,
                             min_opacity: float = 0.01, max_screen_size: float | None = None,
                             scene_extent: float | None = None, reset_opacity: bool = False,
                             max_gaussians: int = 800_000, allow_densify: bool = True,
                             split_normals: t.Tensor | None = None,
                             ) -> tuple[gaussian, t.optim.Optimizer, dict[str, int]]:
    """Clone, split, prune and (optionally) reset opacity, as the reference's function of the
    same name; returns (gaussians, optimizer, {"cloned", "split", "pruned"}). `split_normals`
    (optional, [2 * n_split, 3]) replaces the unit normals of the split offsets: rows [0, n)
    for the first child of each split Gaussian in index order, [n, 2n) for the second."""
    from custom_rasterizer_cuda import _lib

    ensure_densification_state(gaussians)
    if scene_extent is None:
        raise ValueError("scene_extent must be provided.")
    if not gaussians.mu.is_cuda:
        raise RuntimeError("adaptive_density_control needs the Gaussians on a CUDA device")
    stats = {"cloned": 0, "split": 0, "pruned": 0}
    if not allow_densify:
        _reset_stats(gaussians)
        return gaussians, optimizer, stats
    dev = gaussians.mu.device
    n = int(gaussians.mu.shape[0])
    params = [getattr(gaussians, a).detach().contiguous() for a in _ORDER]
    moments = [_group_state(optimizer, a)[2] for a in _ORDER]
    m_in = [st["exp_avg"].contiguous() if st and "exp_avg" in st else None for st in moments]
    v_in = [st["exp_avg_sq"].contiguous() if st and "exp_avg_sq" in st else None
            for st in moments]
    f32 = dict(device=dev, dtype=t.float32)
    grad_accum = gaussians.xyz_grad_accum.detach().to(t.float32).contiguous()
    denom = gaussians.denom.detach().to(t.float32).contiguous()
    radii = gaussians.max_radii2D.detach().to(t.float32).contiguous()
    L = _lib.lib

    def ptrs(ts):
        return (ctypes.c_void_p * 6)(*[x.data_ptr() if x is not None else None for x in ts])

    with t.cuda.device(dev):
        stream = t.cuda.current_stream(dev).cuda_stream
        ws_bytes = L.gs_adc_workspace_size(n)
        ws = t.empty((max(ws_bytes, 1),), device=dev, dtype=t.uint8)
        totals = t.zeros(5, dtype=t.int64, pin_memory=True)
        ev = _lib.Event()

        def plan(prune: bool):
            _lib.check(L.gs_adc_plan(
                n, params[2].data_ptr(), params[3].data_ptr(), grad_accum.data_ptr(),
                denom.data_ptr(), radii.data_ptr(), float(grad_threshold),
                float(percent_dense * scene_extent), float(0.1 * scene_extent),
                float(min_opacity), -1.0 if max_screen_size is None else float(max_screen_size),
                1 if n < max_gaussians else 0, 1 if prune else 0, ws.data_ptr(), ws_bytes,
                totals.data_ptr(), ev.handle, stream))
            ev.synchronize()
            return [int(x) for x in totals.tolist()]

        def apply(tot, z, reset):
            n_out = tot[0] + tot[1] + 2 * tot[3]
            outs = [t.empty((n_out, *p.shape[1:]), **f32) for p in params]
            m_out = [t.empty_like(o) if m is not None else None for o, m in zip(outs, m_in)]
            v_out = [t.empty_like(o) if v is not None else None for o, v in zip(outs, v_in)]
            _lib.check(L.gs_adc_apply(
                n, ws.data_ptr(), ws_bytes, (ctypes.c_longlong * 4)(*tot[:4]), ptrs(params),
                ptrs(m_in), ptrs(v_in), z.data_ptr() if tot[2] else None,
                1 if reset else 0, ptrs(outs), ptrs(m_out), ptrs(v_out), stream))
            return outs, m_out, v_out

        tot = plan(prune=True)
        n_orig, n_clone, n_split, n_child, n_cloned = tot
        stats["split"], stats["cloned"] = n_split, n_cloned
        set_size = (n - n_split) + n_cloned + 2 * n_split  # before the final prune
        if split_normals is not None:
            z = split_normals.to(**f32).contiguous()
            if z.shape != (2 * n_split, 3):
                raise ValueError(f"split_normals must be [{2 * n_split}, 3]")
        else:
            z = t.randn((2 * n_split, 3), **f32) if n_split else t.empty((0, 3), **f32)
        if n_orig + n_clone + 2 * n_child == 0 and set_size > 0:
            # everything would be pruned: the reference keeps the 10% most opaque of the set,
            # then (if asked) resets opacity
            outs, m_out, v_out = apply(plan(prune=False), z, False)
            k = max(1, set_size // 10)
            keep = t.zeros(set_size, dtype=t.bool, device=dev)
            keep[t.topk(t.sigmoid(outs[3].reshape(-1)), k=k).indices] = True
            outs = [o[keep] for o in outs]
            m_out = [m[keep] if m is not None else None for m in m_out]
            v_out = [v[keep] if v is not None else None for v in v_out]
            if reset_opacity:
                outs[3].clamp_(max=math.log(0.01 / (1.0 - 0.01)))
                for mv in (m_out[3], v_out[3]):
                    if mv is not None:
                        mv.zero_()
        else:
            outs, m_out, v_out = apply(tot, z, reset_opacity)
        n_out = int(outs[0].shape[0])
        stats["pruned"] = set_size - n_out
    for a, o, m, v in zip(_ORDER, outs, m_out, v_out):
        new = Parameter(o)
        _replace(optimizer, a, new, m, v)
        setattr(gaussians, a, new)
    gaussians.N = n_out
    _reset_stats(gaussians)
    return gaussians, optimizer, stats

