"""numpy front end of the CPU oracle (gs_oracle.c). TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, as
the checker the CUDA path is compared against; nothing in the product imports it.

All functions take and return numpy arrays in the reference's layouts (float32, int32 for
ids / ranges / counts). `build()` compiles gs_oracle.c with the Makefile beside it.
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import c_float, c_int, c_longlong, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libgs_oracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "gs_oracle.c").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB))
        P = c_void_p
        L.oracle_set_threads.argtypes = [c_int]
        L.oracle_max_threads.restype = c_int
        L.oracle_project.argtypes = [c_int, P, P, P, P, P, c_float, c_float, c_float, c_float,
                                     P, P, P]
        L.oracle_sh.argtypes = [c_int, P, P, P, P, P]
        L.oracle_count.argtypes = [c_int, c_int, c_int, P, P, P]
        L.oracle_count.restype = c_longlong
        L.oracle_bin.argtypes = [c_int, c_int, c_int, P, P, P, c_longlong, P, P, P]
        L.oracle_blend.argtypes = [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P]
        L.oracle_blend_backward.argtypes = [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P,
                                            P, P, P, P]
        L.oracle_sh_backward.argtypes = [c_int, P, P, P, P, P, P, P, P]
        L.oracle_project_backward.argtypes = [c_int, P, P, P, P, P, P, P, c_float, c_float,
                                              c_float, c_float, P, P, P]
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _p(a: np.ndarray):
    return a.ctypes.data_as(c_void_p) if a.size else None


def tiles(H: int, W: int) -> tuple[int, int]:
    return (W + 15) // 16, (H + 15) // 16


def project(mu, q, s, R, t, fx, fy, cx, cy):
    mu, q, s, R, t = map(_f32, (mu, q, s, R, t))
    N = mu.shape[0]
    mean2d = np.zeros((N, 2), np.float32)
    cov2d = np.zeros((N, 3), np.float32)
    depths = np.zeros((N,), np.float32)
    lib().oracle_project(N, _p(mu), _p(q), _p(s), _p(R), _p(t), fx, fy, cx, cy, _p(mean2d),
                         _p(cov2d), _p(depths))
    return mean2d, cov2d, depths


def sh(cam, mu, A, kj):
    cam, mu, A, kj = map(_f32, (cam, mu, A, kj))
    N = mu.shape[0]
    colors = np.zeros((N, 3), np.float32)
    lib().oracle_sh(N, _p(cam), _p(mu), _p(A), _p(kj), _p(colors))
    return colors


def count(mean2d, cov2d, H, W):
    mean2d, cov2d = _f32(mean2d), _f32(cov2d)
    N = mean2d.shape[0]
    counts = np.zeros((N,), np.int32)
    M = lib().oracle_count(N, H, W, _p(mean2d), _p(cov2d), _p(counts))
    return int(M), counts


def bin(mean2d, cov2d, depths, H, W):
    """(keys uint64[M], sorted_ids int32[M], tile_ranges int32[T,2])"""
    mean2d, cov2d, depths = map(_f32, (mean2d, cov2d, depths))
    N = mean2d.shape[0]
    M, _ = count(mean2d, cov2d, H, W)
    tx, ty = tiles(H, W)
    keys = np.zeros((M,), np.uint64)
    ids = np.zeros((M,), np.int32)
    ranges = np.zeros((tx * ty, 2), np.int32)
    lib().oracle_bin(N, H, W, _p(mean2d), _p(cov2d), _p(depths), M, _p(keys), _p(ids),
                     _p(ranges))
    return keys, ids, ranges


def blend(mean2d, cov2d, colors, alpha, sorted_ids, ranges, H, W):
    """(img[H,W,3], final_T[H,W], n_contrib[H,W], ambiguous[H,W] bool)"""
    mean2d, cov2d, colors, alpha = map(_f32, (mean2d, cov2d, colors, alpha))
    sorted_ids, ranges = _i32(sorted_ids), _i32(ranges)
    N = mean2d.shape[0]
    img = np.zeros((H, W, 3), np.float32)
    final_T = np.ones((H, W), np.float32)
    n_contrib = np.zeros((H, W), np.int32)
    amb = np.zeros((H, W), np.uint8)
    lib().oracle_blend(N, H, W, _p(ranges), _p(sorted_ids), _p(mean2d), _p(cov2d), _p(colors),
                       _p(alpha), _p(img), _p(final_T), _p(n_contrib), _p(amb))
    return img, final_T, n_contrib, amb.astype(bool)


def rasterize(depths, mean2d, cov2d, colors, alpha, H, W):
    """Reference `rasterize`: (img, sorted_ids, tile_ranges, final_T, n_contrib) plus
    the sorted keys and the per-pixel ambiguity mask."""
    keys, ids, ranges = bin(mean2d, cov2d, depths, H, W)
    img, final_T, n_contrib, amb = blend(mean2d, cov2d, colors, alpha, ids, ranges, H, W)
    return dict(img=img, sorted_ids=ids, tile_ranges=ranges, final_T=final_T,
                n_contrib=n_contrib, keys=keys, ambiguous=amb)


def rasterize_backward(grad_img, mean2d, cov2d, colors, alpha, sorted_ids, ranges, final_T,
                       n_contrib, H, W):
    """(g_mean2d[N,2], g_cov2d[N,3], g_colors[N,3], g_alpha[N,1], ambiguous[N] bool)"""
    grad_img, mean2d, cov2d, colors, alpha, final_T = map(
        _f32, (grad_img, mean2d, cov2d, colors, alpha, final_T))
    sorted_ids, ranges, n_contrib = map(_i32, (sorted_ids, ranges, n_contrib))
    N = mean2d.shape[0]
    gm = np.zeros((N, 2), np.float32)
    gc = np.zeros((N, 3), np.float32)
    gcol = np.zeros((N, 3), np.float32)
    ga = np.zeros((N, 1), np.float32)
    amb = np.zeros((N,), np.uint8)
    lib().oracle_blend_backward(N, H, W, _p(grad_img), _p(mean2d), _p(cov2d), _p(colors),
                                _p(alpha), _p(sorted_ids), _p(ranges), _p(final_T),
                                _p(n_contrib), _p(gm), _p(gc), _p(gcol), _p(ga), _p(amb))
    return gm, gc, gcol, ga, amb.astype(bool)


def sh_backward(gcol, mu, A, kj, cam):
    gcol, mu, A, kj, cam = map(_f32, (gcol, mu, A, kj, cam))
    N = mu.shape[0]
    gA = np.zeros((N, 3), np.float32)
    gkj = np.zeros((N, 15, 3), np.float32)
    gmu = np.zeros((N, 3), np.float32)
    lib().oracle_sh_backward(N, _p(gcol), _p(mu), _p(A), _p(kj), _p(cam), _p(gA), _p(gkj),
                             _p(gmu))
    return gA, gkj, gmu


def project_backward(gm, gc, mu, q, s, R, t, fx, fy, cx, cy):
    gm, gc, mu, q, s, R, t = map(_f32, (gm, gc, mu, q, s, R, t))
    N = mu.shape[0]
    gmu = np.zeros((N, 3), np.float32)
    gq = np.zeros((N, 4), np.float32)
    gs = np.zeros((N, 3), np.float32)
    lib().oracle_project_backward(N, _p(gm), _p(gc), _p(mu), _p(q), _p(s), _p(R), _p(t), fx,
                                  fy, cx, cy, _p(gmu), _p(gq), _p(gs))
    return gmu, gq, gs


def camera_position(R, t) -> np.ndarray:
    """-R^T t, as the reference wrapper computes it (rasterize.py:43)."""
    R, t = _f32(R), _f32(t)
    return (-(R.T @ t)).astype(np.float32)


def render(mu, q, s, alpha, A, kj, R, t, fx, fy, cx, cy, H, W):
    """Full forward of the reference wrapper; alpha is opacity in (0, 1)."""
    mean2d, cov2d, depths = project(mu, q, s, R, t, fx, fy, cx, cy)
    colors = sh(camera_position(R, t), mu, A, kj)
    out = rasterize(depths, mean2d, cov2d, colors, np.asarray(alpha, np.float32).reshape(-1), H, W)
    out.update(mean2d=mean2d, cov2d=cov2d, depths=depths, colors=colors)
    return out
