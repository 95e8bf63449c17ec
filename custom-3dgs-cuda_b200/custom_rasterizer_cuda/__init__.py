"""Drop-in replacement for the reference's pybind11 module `custom_rasterizer_cuda`.

Same six entry points, argument orders, tensor layouts and error behaviour as
csrc/bindings.cpp:141-151 of the reference; every call validates its tensors here
(RuntimeError with the reference's TORCH_CHECK messages), allocates the outputs with
torch on the inputs' device and forwards raw device pointers to the sm_100a kernels of
libgs3d_b200.so through its C ABI (include/gs3d_b200.h). Work is enqueued on torch's
current CUDA stream (the reference used the legacy default stream).

Differences a caller can observe:
* `SH` and `backwards_SH` read the camera position on the device; the reference copied it
  to the host (csrc/forward/SH.cu:108, csrc/backward/delight_backward.cu:200).
* `rasterize` returns `sorted_ids` as a view of length M of a slightly larger buffer.
* `backwards_projection` returns the derivative of `project`'s quaternion-to-rotation map;
  the reference's hand-written quaternion formula (projection_backward.cu:116-126) is the
  derivative of the transposed rotation under GLM's column-major indexing.
"""

from __future__ import annotations

import threading

import torch

from . import _lib
from ._lib import Event, check, clear_device_errors, device_error_bits, kernel_launches, lib

__all__ = [
    "project",
    "SH",
    "rasterize",
    "backwards_rasterization",
    "backwards_SH",
    "backwards_projection",
    "device_error_bits",
    "clear_device_errors",
    "kernel_launches",
]

TILE = 16
# largest pair capacity the C ABI accepts (gs_rasterize requires pair_capacity < 2^30)
_MAX_PAIRS = (1 << 30) - 1


# ---- input checks (csrc/cuda_check.h:24-47) ------------------------------------------------
def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_input(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    _require(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")
    _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(t.dtype == dtype, f"{name} must be {'FP32' if dtype == torch.float32 else 'int32'}")


def _fp32(t: torch.Tensor, name: str) -> None:
    _check_input(t, name, torch.float32)


def _int32(t: torch.Tensor, name: str) -> None:
    _check_input(t, name, torch.int32)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _tiles(height: int, width: int) -> int:
    return ((width + TILE - 1) // TILE) * ((height + TILE - 1) // TILE)


# ---- projection ----------------------------------------------------------------------------
def project(total_gaussians, mu3d, q3d, s3d, camera_rotation, camera_translation, fx, fy, cx,
            cy):
    """(mean_2d[N,2], cov_2d[N,3], depths[N]); zeros for Gaussians at z <= 0.2."""
    for t, n in ((mu3d, "mu3d"), (q3d, "q3d"), (s3d, "s3d"), (camera_rotation, "camera_rotation"),
                 (camera_translation, "camera_translation")):
        _fp32(t, n)
    N = int(total_gaussians)
    _require(N >= 0, "total_gaussians must be non-negative")
    _require(mu3d.numel() >= 3 * N and q3d.numel() >= 4 * N and s3d.numel() >= 3 * N,
             "mu3d, q3d and s3d must hold total_gaussians rows")
    _require(camera_rotation.numel() >= 9 and camera_translation.numel() >= 3,
             "camera_rotation must be 3x3 and camera_translation 3 elements")
    dev = mu3d.device
    opts = dict(device=dev, dtype=torch.float32)
    mean_2d = torch.empty((N, 2), **opts)
    cov_2d = torch.empty((N, 3), **opts)
    depths = torch.empty((N,), **opts)
    with torch.cuda.device(dev):
        check(lib.gs_project(N, _ptr(mu3d), _ptr(q3d), _ptr(s3d), _ptr(camera_rotation),
                             _ptr(camera_translation), float(fx), float(fy), float(cx),
                             float(cy), _ptr(mean_2d), _ptr(cov_2d), _ptr(depths),
                             _stream(dev)))
    return mean_2d, cov_2d, depths


def backwards_projection(mean_2d_grad, cov_2d_grad, mu, q, s, camera_rotation,
                         camera_translation, fx, fy, cx, cy):
    """(mu_grad[N,3], q_grad[N,4], s_grad[N,3]) with N = mu.size(0)."""
    for t, n in ((mean_2d_grad, "mean_2d_grad"), (cov_2d_grad, "cov_2d_grad"), (mu, "mu"),
                 (q, "q"), (s, "s"), (camera_rotation, "camera_rotation"),
                 (camera_translation, "camera_translation")):
        _fp32(t, n)
    N = int(mu.size(0))
    _require(mean_2d_grad.numel() >= 2 * N and cov_2d_grad.numel() >= 3 * N
             and q.numel() >= 4 * N and s.numel() >= 3 * N, "gradient/parameter sizes")
    dev = mu.device
    opts = dict(device=dev, dtype=torch.float32)
    mu_grad = torch.empty((N, 3), **opts)
    q_grad = torch.empty((N, 4), **opts)
    s_grad = torch.empty((N, 3), **opts)
    with torch.cuda.device(dev):
        check(lib.gs_project_backward(N, _ptr(mean_2d_grad), _ptr(cov_2d_grad), _ptr(mu), _ptr(q),
                                      _ptr(s), _ptr(camera_rotation), _ptr(camera_translation),
                                      float(fx), float(fy), float(cx), float(cy), _ptr(mu_grad),
                                      _ptr(q_grad), _ptr(s_grad), _stream(dev)))
    return mu_grad, q_grad, s_grad


# ---- spherical harmonics -------------------------------------------------------------------
def SH(total_gaussians, camera_position, mu_world, albedo_coeff, illumination_coeff):
    """colors[N,3] = clamp(0.5 + C0*A + sum_k Y_k(dir) k_j[k], 0, 1)."""
    for t, n in ((camera_position, "camera_position"), (mu_world, "mu_world"),
                 (albedo_coeff, "albedo_coeff"), (illumination_coeff, "illumination_coeff")):
        _fp32(t, n)
    _require(camera_position.numel() >= 3, "camera_position must have 3 elements")
    N = int(total_gaussians)
    _require(N >= 0, "total_gaussians must be non-negative")
    _require(mu_world.numel() >= 3 * N and albedo_coeff.numel() >= 3 * N
             and illumination_coeff.numel() >= 45 * N, "inputs must hold total_gaussians rows")
    dev = mu_world.device
    colors = torch.empty((N, 3), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        check(lib.gs_sh_forward(N, _ptr(camera_position), _ptr(mu_world), _ptr(albedo_coeff),
                                _ptr(illumination_coeff), _ptr(colors), _stream(dev)))
    return colors


def backwards_SH(colors_grad, mu, albedo, k_j, camera_position):
    """(albedo_grad[N,3], k_j_grad[N,15,3], mu_grad[N,3]) with N = mu.size(0)."""
    for t, n in ((colors_grad, "colors_grad"), (mu, "mu"), (albedo, "albedo"), (k_j, "k_j"),
                 (camera_position, "camera_position")):
        _fp32(t, n)
    _require(camera_position.numel() >= 3, "camera_position must have 3 elements")
    N = int(mu.size(0))
    _require(colors_grad.numel() >= 3 * N and albedo.numel() >= 3 * N and k_j.numel() >= 45 * N,
             "inputs must hold N rows")
    dev = mu.device
    opts = dict(device=dev, dtype=torch.float32)
    albedo_grad = torch.empty((N, 3), **opts)
    k_j_grad = torch.empty((N, 15, 3), **opts)
    mu_grad = torch.empty((N, 3), **opts)
    with torch.cuda.device(dev):
        check(lib.gs_sh_backward(N, _ptr(colors_grad), _ptr(mu), _ptr(albedo), _ptr(k_j),
                                 _ptr(camera_position), _ptr(albedo_grad), _ptr(k_j_grad),
                                 _ptr(mu_grad), _stream(dev)))
    return albedo_grad, k_j_grad, mu_grad


# ---- rasterization -------------------------------------------------------------------------
class _PairCapacity:
    """Remembers the pair count M of earlier calls per (N, H, W, binning mode) to size the next
    call's pair buffers; a call whose M exceeds the guess is re-run with exactly M."""

    def __init__(self) -> None:
        self._last: dict[tuple[int, int, int, int], int] = {}
        self._lock = threading.Lock()

    def guess(self, n: int, h: int, w: int, mode: int = 0) -> int:
        with self._lock:
            m = self._last.get((n, h, w, mode))
        if m is None:
            return min(8 * n + 4096, (1 << 30) - 1)
        return min(m + m // 8 + 4096, (1 << 30) - 1)

    def update(self, n: int, h: int, w: int, m: int, mode: int = 0) -> None:
        with self._lock:
            self._last[(n, h, w, mode)] = m


_capacity = _PairCapacity()
_events = threading.local()


def _m_event() -> Event:
    ev = getattr(_events, "ev", None)
    if ev is None:
        ev = _events.ev = Event()
    return ev


def _empty_raster(device, height, width):
    T = _tiles(height, width)
    return (
        torch.zeros((height, width, 3), device=device, dtype=torch.float32),
        torch.empty((0,), device=device, dtype=torch.int32),
        torch.zeros((T, 2), device=device, dtype=torch.int32),
        torch.ones((height, width), device=device, dtype=torch.float32),
        torch.zeros((height, width), device=device, dtype=torch.int32),
    )


def rasterize(num_gaussians, depths, mean_2d, cov_2d, colors, alpha, height, width):
    """(rendered_img[H,W,3], sorted_ids[M], tile_ranges[T,2], final_T[H,W], n_contrib[H,W])."""
    N, H, W = int(num_gaussians), int(height), int(width)
    if N == 0:
        return _empty_raster(mean_2d.device, H, W)
    for t, n in ((depths, "depths"), (mean_2d, "mean_2d"), (cov_2d, "cov_2d"),
                 (colors, "colors"), (alpha, "alpha")):
        _fp32(t, n)
    _require(mean_2d.dim() == 2 and mean_2d.size(0) == N and mean_2d.size(1) == 2,
             "mean_2d must have shape (N, 2)")
    _require(cov_2d.dim() == 2 and cov_2d.size(0) == N and cov_2d.size(1) == 3,
             "cov_2d must have shape (N, 3) upper-triangular [a, b, c]")
    _require(colors.dim() == 2 and colors.size(0) == N and colors.size(1) == 3,
             "colors must have shape (N, 3)")
    _require(depths.numel() == N, "depths must have N elements")
    _require(alpha.numel() == N, "alpha must have N elements")
    _require(H > 0 and W > 0, "height and width must be positive")
    dev = mean_2d.device
    T = _tiles(H, W)
    cap = _capacity.guess(N, H, W)
    with torch.cuda.device(dev):
        stream = _stream(dev)
        f32 = dict(device=dev, dtype=torch.float32)
        i32 = dict(device=dev, dtype=torch.int32)
        img = torch.empty((H, W, 3), **f32)
        final_T = torch.empty((H, W), **f32)
        n_contrib = torch.empty((H, W), **i32)
        tile_ranges = torch.empty((T, 2), **i32)
        m_host = torch.empty((1,), dtype=torch.int32, pin_memory=True)
        ev = _m_event()
        for _attempt in range(2):
            ws_bytes = lib.gs_rasterize_workspace_size(N, H, W, cap)
            ws = torch.empty((ws_bytes,), device=dev, dtype=torch.uint8)
            sorted_ids = torch.empty((cap,), **i32)
            check(lib.gs_rasterize(N, H, W, _ptr(depths), _ptr(mean_2d), _ptr(cov_2d),
                                   _ptr(colors), _ptr(alpha), ws.data_ptr(), ws_bytes, cap,
                                   _ptr(img), _ptr(sorted_ids), _ptr(tile_ranges),
                                   _ptr(final_T), _ptr(n_contrib), None, m_host.data_ptr(),
                                   ev.handle, stream))
            ev.synchronize()
            M = int(m_host[0])
            _capacity.update(N, H, W, M)
            if M <= cap:
                return img, sorted_ids[:M], tile_ranges, final_T, n_contrib
            if M > _MAX_PAIRS:
                raise RuntimeError(
                    f"rasterize: {M} (tile, Gaussian) pairs exceed the supported maximum of "
                    f"{_MAX_PAIRS}; reduce the number of Gaussians or the image size")
            cap = M
        raise RuntimeError("pair count kept growing between attempts")


def backwards_rasterization(grad_output, mean_2d, cov_2d, colors, alpha, sorted_ids,
                            tile_ranges, final_T, n_contrib, num_gaussians, height, width):
    """(grad_mean_2d[N,2], grad_cov_2d[N,3] = dL/dSigma2, grad_colors[N,3], grad_alpha[N,1])."""
    for t, n in ((grad_output, "grad_output"), (mean_2d, "mean_2d"), (cov_2d, "cov_2d"),
                 (colors, "colors"), (alpha, "alpha"), (final_T, "final_T")):
        _fp32(t, n)
    for t, n in ((sorted_ids, "sorted_ids"), (tile_ranges, "tile_ranges"),
                 (n_contrib, "n_contrib")):
        _int32(t, n)
    N, H, W = int(num_gaussians), int(height), int(width)
    _require(mean_2d.dim() == 2 and mean_2d.size(0) == N and mean_2d.size(1) == 2,
             "mean_2d must have shape (N, 2)")
    _require(cov_2d.dim() == 2 and cov_2d.size(0) == N and cov_2d.size(1) == 3,
             "cov_2d must have shape (N, 3)")
    _require(colors.dim() == 2 and colors.size(0) == N and colors.size(1) == 3,
             "colors must have shape (N, 3)")
    _require(alpha.numel() == N, "alpha must have N elements")
    _require(final_T.numel() == H * W, "final_T must have H*W elements")
    _require(n_contrib.numel() == H * W, "n_contrib must have H*W elements")
    _require(grad_output.numel() == H * W * 3, "grad_output must have H*W*3 elements")
    _require(tile_ranges.numel() >= 2 * _tiles(H, W), "tile_ranges must have T rows")
    dev = mean_2d.device
    f32 = dict(device=dev, dtype=torch.float32)
    grad_mean_2d = torch.zeros((N, 2), **f32)
    grad_cov_2d = torch.zeros((N, 3), **f32)
    grad_colors = torch.zeros((N, 3), **f32)
    grad_alpha = torch.zeros((N, 1), **f32)
    if N == 0:
        return grad_mean_2d, grad_cov_2d, grad_colors, grad_alpha
    with torch.cuda.device(dev):
        ws_bytes = lib.gs_rasterize_backward_workspace_size(N)
        ws = torch.empty((ws_bytes,), device=dev, dtype=torch.uint8)
        check(lib.gs_rasterize_backward(N, H, W, _ptr(grad_output), _ptr(mean_2d), _ptr(cov_2d),
                                        _ptr(colors), _ptr(alpha), _ptr(sorted_ids),
                                        _ptr(tile_ranges), _ptr(final_T), _ptr(n_contrib),
                                        ws.data_ptr(), ws_bytes, _ptr(grad_mean_2d),
                                        _ptr(grad_cov_2d), _ptr(grad_colors), _ptr(grad_alpha),
                                        _stream(dev)))
    return grad_mean_2d, grad_cov_2d, grad_colors, grad_alpha
