"""Fused render path over gs_render_forward / gs_render_backward (include/gs3d_b200.h).

`render_forward` renders one view straight from the Gaussian parameters and returns the
image, the screen radii and a `RenderState` that `render_backward` needs; `render_backward`
returns (or accumulates into given buffers) the gradients of all six parameters. Outputs are
identical to chaining project -> SH -> rasterize and their backwards, as the reference wrapper
does (gaussian_splatting/rasterizer/rasterize.py:43-117).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _MAX_PAIRS, _capacity, _ptr, _stream, _tiles
from ._lib import check, lib


# Scenes whose worst case of (tile, Gaussian) pairs -- every Gaussian in every tile, N * T --
# stays within this many pairs get pair buffers for that worst case (16 bytes per pair of
# workspace), so no call can overflow and the host never waits for the pair count.
_WORST_CASE_PAIRS = 1 << 22


@dataclass
class RenderState:
    workspace: torch.Tensor
    capacity: int
    sorted_ids: torch.Tensor   # [capacity]; the first M are valid
    tile_ranges: torch.Tensor
    final_T: torch.Tensor
    n_contrib: torch.Tensor
    height: int
    width: int
    backward_flags: int = 0    # GS_RENDER_CONCURRENT when the forward was given it
    m_host: torch.Tensor | None = None  # pinned int32: M, valid once m_event has completed
    m_event: object = None
    _pairs: int | None = None
    _key: tuple | None = None

    @property
    def pairs(self) -> int:
        """M, the number of (tile, Gaussian) pairs (waits for it on first use)."""
        if self._pairs is None:
            self.m_event.synchronize()
            self._pairs = int(self.m_host[0])
            n, h, w, mode = self._key
            _capacity.update(n, h, w, self._pairs, mode)
        return self._pairs

    def overflowed(self) -> bool:
        """True if M exceeded the pair buffers: the image and the state are then unusable and
        the view must be rendered again (waits for M on first use)."""
        return self.pairs > self.capacity


def render_forward(mu, q, s, opacity, albedo, k_j, R, t, cam_pos, fx, fy, cx, cy, height,
                   width, tight_bins: bool = False, concurrent: bool = False,
                   defer_check: bool = False, capacity: int | None = None):
    """(img[H,W,3], radii[N], RenderState). `opacity` is post-sigmoid, N or [N,1].
    tight_bins: bin splats only into tiles where they can pass the opacity test (same image
    and gradients, shorter tile lists; the state's lists then differ from the reference's).
    concurrent: the caller overlaps several views on streams; the blend kernels (this one and
    the state's backward) use their throughput variants (GS_RENDER_CONCURRENT).
    Pair buffers are sized for the scene's worst case when that is small (no host wait at
    all), otherwise from the pair count of earlier calls (+12.5%) or `capacity`. Then, by
    default, the call waits for the pair count and renders again with exactly M if the guess
    was short; with defer_check=True it returns at once and the caller must ask
    `state.overflowed()` before using the image or the state, and render again (with
    capacity=state.pairs) if it is true."""
    N, H, W = int(mu.shape[0]), int(height), int(width)
    dev = mu.device
    T = _tiles(H, W)
    f32 = dict(device=dev, dtype=torch.float32)
    i32 = dict(device=dev, dtype=torch.int32)
    img = torch.empty((H, W, 3), **f32)
    final_T = torch.empty((H, W), **f32)
    n_contrib = torch.empty((H, W), **i32)
    tile_ranges = torch.empty((T, 2), **i32)
    radii = torch.empty((N,), **f32)
    mode = 1 if tight_bins else 0
    flags = mode | (2 if concurrent else 0)
    worst = N * T
    safe = worst <= _WORST_CASE_PAIRS
    if capacity is not None:
        cap = int(capacity)
    else:
        cap = worst if safe else _capacity.guess(N, H, W, mode)
    key = (N, H, W, mode)
    with torch.cuda.device(dev):
        stream = _stream(dev)
        slots = _pair_count_slot()
        for _attempt in range(2):
            slot, m_host, ev = slots.take()
            ws_bytes = lib.gs_render_workspace_size(N, H, W, cap)
            ws = torch.empty((ws_bytes,), device=dev, dtype=torch.uint8)
            sorted_ids = torch.empty((max(cap, 1),), **i32)
            check(lib.gs_render_forward(
                N, H, W, _ptr(mu), _ptr(q), _ptr(s), _ptr(opacity), _ptr(albedo), _ptr(k_j),
                _ptr(R), _ptr(t), _ptr(cam_pos), float(fx), float(fy), float(cx), float(cy),
                ws.data_ptr(), ws_bytes, cap, _ptr(img), sorted_ids.data_ptr(),
                _ptr(tile_ranges), _ptr(final_T), _ptr(n_contrib), _ptr(radii),
                m_host.data_ptr(), ev.handle, flags, stream))
            state = RenderState(ws, cap, sorted_ids, tile_ranges, final_T, n_contrib, H, W,
                                flags & 2, m_host, ev, None, key)
            slots.own(slot, state)
            if safe or defer_check or not state.overflowed():
                return img, radii, state
            M = state.pairs
            if M > _MAX_PAIRS:
                raise RuntimeError(
                    f"render: {M} (tile, Gaussian) pairs exceed the supported maximum of "
                    f"{_MAX_PAIRS}; reduce the number of Gaussians or the image size")
            cap = M
    raise RuntimeError("pair count kept growing between attempts")


class _PairCountSlots:
    """Pinned host words that receive each render's pair count, with an event per word. A word
    is reused round-robin; before that, the render that used it last is made to read its count
    (its copy long finished by then), so a state never sees another render's count and no
    copy ever lands in memory that has been handed to someone else."""

    def __init__(self, n: int = 256) -> None:
        import threading
        import weakref

        self._weakref = weakref.ref
        self.buf = torch.empty((n,), dtype=torch.int32, pin_memory=True)
        self.events: list = [None] * n
        self.owners: list = [None] * n
        self.next = 0
        self.lock = threading.Lock()

    def take(self):
        from ._lib import Event

        with self.lock:
            k = self.next
            self.next = (k + 1) % self.buf.numel()
            owner = self.owners[k]() if self.owners[k] is not None else None
            if owner is not None:
                owner.pairs  # resolves its count before the word is reused
            ev = self.events[k]
            if ev is None:
                ev = self.events[k] = Event()
            else:
                ev.synchronize()
            return k, self.buf[k:k + 1], ev

    def own(self, k: int, state) -> None:
        self.owners[k] = self._weakref(state)


_slots = None


def _pair_count_slot():
    global _slots
    if _slots is None:
        _slots = _PairCountSlots()
    return _slots


def render_backward(state: RenderState, grad_img, mu, q, s, albedo, k_j, R, t, cam_pos, fx, fy,
                    cx, cy, want_mean2d_grad: bool = True, out=None, stats=None,
                    accum_wait=None, accum_done=None, accumulate=None):
    """Gradients (mu, q, s, opacity[N], albedo, k_j, mean2d or None). With `out` (a tuple of
    the first six buffers) the gradients are added into those buffers instead. `stats` =
    (norm_sum[N], count[N], norm_max[N], scale_x, scale_y) updates the densification
    statistics in the same pass. `accum_wait` / `accum_done` (`_lib.Event` or None) order the
    kernel that writes `out` and `stats` after / before other streams' writes to them.
    `accumulate=False` with `out` overwrites the six buffers instead (every element written);
    the statistics are always added to."""
    N = int(mu.shape[0])
    dev = mu.device
    f32 = dict(device=dev, dtype=torch.float32)
    if accumulate is None:
        accumulate = out is not None
    if out is None:
        accumulate = False
        out = (torch.empty((N, 3), **f32), torch.empty((N, 4), **f32), torch.empty((N, 3), **f32),
               torch.empty((N,), **f32), torch.empty((N, 3), **f32),
               torch.empty((N, 15, 3), **f32))
    g_mean2d = torch.empty((N, 2), **f32) if want_mean2d_grad else None
    grad_img = grad_img.contiguous()
    with torch.cuda.device(dev):
        ws_bytes = lib.gs_render_backward_workspace_size(N)
        ws = torch.empty((ws_bytes,), device=dev, dtype=torch.uint8)
        check(lib.gs_render_backward(
            N, state.height, state.width, _ptr(grad_img), _ptr(mu), _ptr(q), _ptr(s),
            _ptr(albedo), _ptr(k_j), _ptr(R), _ptr(t), _ptr(cam_pos), float(fx), float(fy),
            float(cx), float(cy), state.workspace.data_ptr(), state.capacity,
            state.sorted_ids.data_ptr(), _ptr(state.tile_ranges), _ptr(state.final_T),
            _ptr(state.n_contrib), ws.data_ptr(), ws_bytes, *(_ptr(o) for o in out),
            _ptr(g_mean2d), 1 if accumulate else 0,
            *((_ptr(stats[0]), _ptr(stats[1]), _ptr(stats[2]), float(stats[3]), float(stats[4]))
              if stats is not None else (None, None, None, 0.0, 0.0)),
            accum_wait.handle if accum_wait is not None else None,
            accum_done.handle if accum_done is not None else None,
            state.backward_flags, _stream(dev)))
    return (*out, g_mean2d)


def backward_workspace_bytes(n: int) -> int:
    """Bytes of one view's render_backward_blend workspace for n Gaussians."""
    return int(lib.gs_render_backward_workspace_size(int(n)))


def backward_workspace(n: int, device) -> torch.Tensor:
    """A workspace for one view's render_backward_blend sums (3 float4 per Gaussian)."""
    return torch.empty((backward_workspace_bytes(n),), device=device, dtype=torch.uint8)


def render_backward_blend(state: RenderState, grad_img, n: int, workspace=None) -> torch.Tensor:
    """First half of render_backward for one of several views: the blend backward of the view
    rendered into `state`, leaving its per-Gaussian sums in `workspace` (backward_workspace(n),
    allocated when None), which is returned for render_backward_views."""
    dev = state.final_T.device
    if workspace is None:
        workspace = backward_workspace(n, dev)
    grad_img = grad_img.contiguous()
    with torch.cuda.device(dev):
        check(lib.gs_render_backward_blend(
            int(n), state.height, state.width, _ptr(grad_img), state.workspace.data_ptr(),
            state.capacity, state.sorted_ids.data_ptr(), _ptr(state.tile_ranges),
            _ptr(state.final_T), _ptr(state.n_contrib), workspace.data_ptr(),
            workspace.numel(), state.backward_flags, _stream(dev)))
    return workspace


def render_backward_views(views, mu, q, s, albedo, k_j, out, accumulate: bool = False,
                          stats=None) -> None:
    """Second half of render_backward for several views at once: `views` is a list of
    (workspace from render_backward_blend, R, t, cam_pos, fx, fy, cx, cy, stat_scale_x,
    stat_scale_y); the six gradient buffers `out` get the views' gradients summed in list order,
    after their own values (`accumulate`) or zero, with the same bits as one render_backward per
    view accumulating in that order. `stats` = (norm_sum, count, norm_max) as in render_backward,
    each view with its own scales. Up to GS_MAX_VIEWS_PER_CALL views per launch."""
    from ._lib import GS_MAX_VIEWS_PER_CALL, ViewSums

    N = int(mu.shape[0])
    dev = mu.device
    st = (None, None, None) if stats is None else tuple(_ptr(x) for x in stats[:3])
    with torch.cuda.device(dev):
        for c0 in range(0, len(views), GS_MAX_VIEWS_PER_CALL):
            chunk = views[c0:c0 + GS_MAX_VIEWS_PER_CALL]
            arr = (ViewSums * len(chunk))()
            for k, (ws, R, t, cam, fx, fy, cx, cy, sx, sy) in enumerate(chunk):
                arr[k] = ViewSums(ws.data_ptr(), ws.numel() * ws.element_size(), _ptr(R),
                                  _ptr(t), _ptr(cam), float(fx), float(fy), float(cx),
                                  float(cy), float(sx), float(sy))
            check(lib.gs_render_backward_gaussians(
                N, len(chunk), ctypes.addressof(arr), _ptr(mu), _ptr(q), _ptr(s), _ptr(albedo),
                _ptr(k_j), *(_ptr(o) for o in out), 1 if (accumulate or c0 > 0) else 0, *st,
                _stream(dev)))
