"""numpy restatement of the reference's adaptive density control. TEST INFRASTRUCTURE ONLY.

Only tests/ use this module, as the checker the CUDA density control is compared against;
nothing in the product imports it. It follows gaussian_splatting/utils/adc.py of the
reference: the gradient statistic (:345-346), clone (:197-228), split (:231-296), the final
prune (:363-377) with its keep-the-most-opaque fallback, the opacity reset (:299-315) and the optimizer-state edits (:120-165), with
the split offsets taken as `z * std` for given unit normals `z` (the reference draws them with
`t.normal(mean=0, std)`, :262-263). Its agreement with the reference is pinned by
tests/golden/ref_adc_*.npz, which the reference itself produced (tests/golden/make_adc_golden.py).

Arrays are float32 in the reference layouts: mu[N,3], q[N,4], s[N,3], alpha[N,1], A[N,3],
k_j[N,15,3]; moments have the parameter's shape.
"""

from __future__ import annotations

import math

import numpy as np

NAMES = ("mu", "q", "s", "alpha", "A", "k_j")
F32 = np.float32


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return (F32(1.0) / (F32(1.0) + np.exp(-x, dtype=F32))).astype(F32)


def _rotation(q: np.ndarray) -> np.ndarray:
    """Rotation matrices of quaternions (w, x, y, z), normalised with a 1e-12 floor."""
    n = np.sqrt((q * q).sum(axis=1, dtype=F32), dtype=F32)
    qn = (q / np.maximum(n, F32(1e-12))[:, None]).astype(F32)
    w, x, y, z = qn[:, 0], qn[:, 1], qn[:, 2], qn[:, 3]
    one, two = F32(1.0), F32(2.0)
    r = np.empty((q.shape[0], 3, 3), F32)
    r[:, 0, 0] = one - two * (y * y + z * z)
    r[:, 0, 1] = two * (x * y - w * z)
    r[:, 0, 2] = two * (x * z + w * y)
    r[:, 1, 0] = two * (x * y + w * z)
    r[:, 1, 1] = one - two * (x * x + z * z)
    r[:, 1, 2] = two * (y * z - w * x)
    r[:, 2, 0] = two * (x * z - w * y)
    r[:, 2, 1] = two * (y * z + w * x)
    r[:, 2, 2] = one - two * (x * x + y * y)
    return r


def classify(s, alpha, grad_accum, denom, max_radii, *, grad_threshold, percent_dense,
             scene_extent, min_opacity, max_screen_size, densify, prune):
    """Per-Gaussian decisions: (clone, split, keep_original, keep_clone, keep_children)."""
    grads = (grad_accum.reshape(-1) / np.maximum(denom.reshape(-1), F32(1.0))).astype(F32)
    grads = np.nan_to_num(grads, nan=0.0).astype(F32)
    scales = np.exp(s, dtype=F32)
    ms = scales.max(axis=1)
    thr = F32(grad_threshold)
    pd_line = F32(percent_dense * scene_extent)
    big_line = F32(0.1 * scene_extent)
    clone = densify & (grads >= thr) & (ms <= pd_line)
    split = densify & (grads >= thr) & (ms > pd_line)
    op = _sigmoid(alpha.reshape(-1))
    child_s = np.log((scales / F32(1.6)).astype(F32), dtype=F32)
    ms_child = np.exp(child_s, dtype=F32).max(axis=1)

    def pruned(msx, radii):
        out = (op < F32(min_opacity)) | (msx > big_line)
        if max_screen_size is not None:
            out = out | (radii > F32(max_screen_size))
        return out & prune

    zero = np.zeros_like(max_radii)
    keep_orig = ~split & ~pruned(ms, max_radii)
    keep_clone = clone & ~pruned(ms, zero)
    keep_child = split & ~pruned(ms_child, zero)
    return clone, split, keep_orig, keep_clone, keep_child


def adaptive_density_control(params: dict, exp_avg: dict, exp_avg_sq: dict, grad_accum, denom,
                             max_radii, z, *, grad_threshold=0.00005, percent_dense=0.01,
                             min_opacity=0.01, max_screen_size=None, scene_extent,
                             reset_opacity=False, max_gaussians=800_000, allow_densify=True):
    """Returns (params, exp_avg, exp_avg_sq, counts) after one density-control call; counts =
    (cloned, split, pruned) as the reference reports them. `z` holds 2 * n_split unit normals
    [.., 3]: rows [0, n) for the first child of each split Gaussian, [n, 2n) for the second."""
    if not allow_densify:
        return dict(params), dict(exp_avg), dict(exp_avg_sq), (0, 0, 0)
    n = params["mu"].shape[0]
    densify = n < max_gaussians
    clone, split, keep_orig, keep_clone, keep_child = classify(
        params["s"], params["alpha"], grad_accum, denom, max_radii,
        grad_threshold=grad_threshold, percent_dense=percent_dense, scene_extent=scene_extent,
        min_opacity=min_opacity, max_screen_size=max_screen_size, densify=densify, prune=True)
    n_split = int(split.sum())
    scales = np.exp(params["s"][split], dtype=F32)
    stds = np.concatenate([scales, scales])
    samples = (F32(0.0) + z[:2 * n_split].astype(F32) * stds).astype(F32)
    rots = np.concatenate([_rotation(params["q"][split])] * 2)
    child_mu = (np.einsum("nij,nj->ni", rots, samples).astype(F32)
                + np.concatenate([params["mu"][split]] * 2)).astype(F32)
    child_s = np.log((np.concatenate([scales] * 2) / F32(1.6)).astype(F32), dtype=F32)
    # set after clone and split: [originals not split, clones, children]; pruned in place
    total_set = int((~split).sum() + clone.sum() + 2 * n_split)
    kept = int(keep_orig.sum() + keep_clone.sum() + 2 * keep_child.sum())
    kc = np.concatenate([keep_child[split]] * 2)  # children in split order, two rounds
    if kept == 0 and total_set > 0:
        # every Gaussian would be pruned: keep the max(1, n // 10) most opaque of the set
        # (:371-376), in set order
        keep_orig, keep_clone, kc = ~split, clone.copy(), np.ones(2 * n_split, bool)
        set_alpha = np.concatenate([params["alpha"][~split], params["alpha"][clone],
                                    np.concatenate([params["alpha"][split]] * 2)]).reshape(-1)
        k = max(1, total_set // 10)
        top = np.zeros(total_set, bool)
        top[np.argsort(-_sigmoid(set_alpha), kind="stable")[:k]] = True
        n_o, n_c = int(keep_orig.sum()), int(keep_clone.sum())
        keep_orig[np.flatnonzero(keep_orig)] = top[:n_o]
        keep_clone[np.flatnonzero(keep_clone)] = top[n_o:n_o + n_c]
        kc = top[n_o + n_c:]
        kept = k
    out_p, out_m, out_v = {}, {}, {}
    for name in NAMES:
        p = params[name]
        if name == "mu":
            child = child_mu
        elif name == "s":
            child = child_s
        else:
            child = np.concatenate([p[split]] * 2)
        out_p[name] = np.concatenate([p[keep_orig], p[keep_clone], child[kc]]).astype(F32)
        for src, dst in ((exp_avg, out_m), (exp_avg_sq, out_v)):
            m = src[name]
            pad = np.zeros((int(keep_clone.sum() + kc.sum()),) + m.shape[1:], F32)
            dst[name] = np.concatenate([m[keep_orig], pad]).astype(F32)
    if reset_opacity:
        logit = F32(math.log(0.01 / (1.0 - 0.01)))
        out_p["alpha"] = np.minimum(out_p["alpha"], logit)
        out_m["alpha"] = np.zeros_like(out_m["alpha"])
        out_v["alpha"] = np.zeros_like(out_v["alpha"])
    counts = (int(clone.sum()), n_split, total_set - kept)
    return out_p, out_m, out_v, counts
