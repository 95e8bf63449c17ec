"""gs_rasterize_noalloc, the allocation-free rasterize for callers that cannot allocate device
memory at render time (plugins handed only their buffers, processes whose device memory is
owned by another allocator, per-frame paths that must avoid cudaMalloc's synchronisation).

It is called through the C ABI and compared with the workspace-taking entry point
(`custom_rasterizer_cuda.rasterize` -> gs_rasterize) on consecutive calls with different
inputs, so stale contents of the shared fixed scratch would show up as a mismatch. This file
is collected last; it must pass alone in a fresh process and after the other tests.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch


def _inputs(crc, sc, view, dev):
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    R, t = view.R.to(dev).contiguous(), view.T.to(dev).contiguous()
    mean2d, cov2d, depths = crc.project(sc.N, mu, q, s, R, t, view.fx, view.fy, view.cx, view.cy)
    colors = crc.SH(sc.N, (-(R.T @ t)).contiguous(), mu, A, kj)
    return depths, mean2d, cov2d, colors, torch.sigmoid(al).contiguous()


def _noalloc(lib, N, H, W, depths, mean2d, cov2d, colors, alpha, capacity, dev):
    T = ((W + 15) // 16) * ((H + 15) // 16)
    img = torch.empty((H, W, 3), device=dev)
    ids = torch.empty((capacity,), device=dev, dtype=torch.int32)
    ranges = torch.empty((T, 2), device=dev, dtype=torch.int32)
    final_T = torch.empty((H, W), device=dev)
    n_contrib = torch.empty((H, W), device=dev, dtype=torch.int32)
    m_dev = torch.full((1,), -1, device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.gs_rasterize_noalloc(N, H, W, depths.data_ptr(), mean2d.data_ptr(),
                                  cov2d.data_ptr(), colors.data_ptr(), alpha.data_ptr(), capacity,
                                  img.data_ptr(), ids.data_ptr(), ranges.data_ptr(),
                                  final_T.data_ptr(), n_contrib.data_ptr(), m_dev.data_ptr(),
                                  stream)
    torch.cuda.synchronize(dev)
    return rc, img, ids, ranges, final_T, n_contrib, int(m_dev.item())


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(crc, cuda_device):
    from custom_rasterizer_cuda import _lib
    from gs3d_b200 import scenes

    dev = cuda_device
    sc0 = scenes.config0(0)
    sc1 = scenes.config2(4, n=30_000)
    cases = [(sc0, sc0.views[0]),
             (sc1, scenes.pinhole((0.0, 0.0, 8.0), 400, 250, 310.0)),
             (sc0, scenes.pinhole((0.5, 0.3, 3.5), 150, 100, 110.0))]
    for sc, view in cases:
        H, W = view.height, view.width
        inp = _inputs(crc, sc, view, dev)
        img_r, ids_r, ranges_r, T_r, nc_r = crc.rasterize(sc.N, *inp, H, W)
        M = ids_r.numel()
        rc, img, ids, ranges, final_T, n_contrib, m = _noalloc(_lib.lib, sc.N, H, W, *inp,
                                                               M + 1000, dev)
        assert rc == _lib.GS_OK, _lib.lib.gs_last_error()
        assert m == M
        assert torch.equal(ids[:M], ids_r)
        assert torch.equal(ranges, ranges_r)
        assert torch.equal(n_contrib, nc_r)
        # the same kernels run in both entry points, so the blend is bit-identical
        assert torch.equal(final_T, T_r)
        assert torch.equal(img, img_r)
    assert crc.device_error_bits() == 0


@pytest.mark.gpu
def test_noalloc_overflow_reports_m_and_a_retry_matches(crc, cuda_device):
    """A capacity below M: the call still returns GS_OK and reports M through pair_count_dev
    (the outputs are not written); a second call with capacity M matches gs_rasterize."""
    from custom_rasterizer_cuda import _lib
    from gs3d_b200 import scenes

    dev = cuda_device
    sc = scenes.config2(6, n=20_000)
    view = scenes.pinhole((0.0, 0.0, 8.0), 320, 200, 250.0)
    H, W = view.height, view.width
    inp = _inputs(crc, sc, view, dev)
    img_r, ids_r, ranges_r, T_r, nc_r = crc.rasterize(sc.N, *inp, H, W)
    M = ids_r.numel()
    assert M > 100
    rc, *_, m = _noalloc(_lib.lib, sc.N, H, W, *inp, M // 3, dev)
    assert rc == _lib.GS_OK and m == M
    rc, img, ids, ranges, final_T, n_contrib, m = _noalloc(_lib.lib, sc.N, H, W, *inp, M, dev)
    assert rc == _lib.GS_OK and m == M
    assert torch.equal(ids, ids_r) and torch.equal(ranges, ranges_r)
    assert torch.equal(n_contrib, nc_r) and torch.equal(final_T, T_r) and torch.equal(img, img_r)
    assert crc.device_error_bits() == 0


@pytest.mark.gpu
def test_noalloc_zero_gaussians_and_a_layout_just_under_the_limit(crc, cuda_device):
    """N == 0 gives the reference's empty render (zero image, final_T = 1, zero ranges and
    counts) even after a call that left other contents in the shared scratch; a layout within
    64 KiB of the 16 MiB limit is accepted and matches gs_rasterize."""
    from custom_rasterizer_cuda import _lib
    from gs3d_b200 import scenes

    dev = cuda_device
    L = _lib.lib
    z = torch.zeros((0, 3), device=dev)
    rc, img, ids, ranges, final_T, n_contrib, m = _noalloc(L, 0, 40, 70, z, z, z, z, z, 16, dev)
    assert rc == _lib.GS_OK and m == 0
    assert float(img.abs().sum()) == 0.0 and bool((final_T == 1).all())
    assert int(ranges.abs().sum()) == 0 and int(n_contrib.abs().sum()) == 0

    limit = 16 << 20
    sc = scenes.config2(7, n=65_536)
    view = scenes.pinhole((0.0, 0.0, 8.0), 1024, 1024, 800.0)
    H, W = view.height, view.width
    lo, hi = 0, 1 << 24  # largest pair capacity whose layout fits the fixed scratch
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if L.gs_rasterize_workspace_size(sc.N, H, W, mid) <= limit else (lo, mid)
    cap = lo
    assert limit - L.gs_rasterize_workspace_size(sc.N, H, W, cap) < 64 << 10
    inp = _inputs(crc, sc, view, dev)
    img_r, ids_r, ranges_r, T_r, nc_r = crc.rasterize(sc.N, *inp, H, W)
    M = ids_r.numel()
    assert 0 < M <= cap
    rc, img, ids, ranges, final_T, n_contrib, m = _noalloc(L, sc.N, H, W, *inp, cap, dev)
    assert rc == _lib.GS_OK, L.gs_last_error()
    assert m == M and torch.equal(ids[:M], ids_r) and torch.equal(ranges, ranges_r)
    assert torch.equal(n_contrib, nc_r) and torch.equal(final_T, T_r) and torch.equal(img, img_r)
    rc, *_ = _noalloc(L, sc.N, H, W, *inp, cap + 4096, dev)
    assert rc == _lib.GS_ERR_CAPACITY
    assert crc.device_error_bits() == 0


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    """Checked on the host before any GPU work, so this runs without a GPU too."""
    from custom_rasterizer_cuda import _lib

    L = _lib.lib
    rc = L.gs_rasterize_noalloc(1_000_000, 1080, 1920, 1, 1, 1, 1, 1, 8_000_000, 1, 1, 1, 1, 1,
                                1, None)
    assert rc == _lib.GS_ERR_CAPACITY
    msg = L.gs_last_error().decode()
    assert "fixed scratch holds 16777216 bytes" in msg and "gs_rasterize" in msg


def test_noalloc_requires_the_pair_count_pointer():
    """Without pair_count_dev a caller could not tell an overflowed call (outputs unwritten)
    from a complete one, so NULL is rejected on the host."""
    from custom_rasterizer_cuda import _lib

    L = _lib.lib
    rc = L.gs_rasterize_noalloc(16, 32, 32, 1, 1, 1, 1, 1, 64, 1, 1, 1, 1, 1, None, None)
    assert rc == _lib.GS_ERR_INVALID_ARG
    assert "pair_count_dev" in L.gs_last_error().decode()
