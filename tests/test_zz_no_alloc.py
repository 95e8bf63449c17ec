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
        np.testing.assert_allclose(final_T.cpu().numpy(), T_r.cpu().numpy(), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(img.cpu().numpy(), img_r.cpu().numpy(), rtol=1e-5, atol=1e-6)
    assert crc.device_error_bits() == 0


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    """Checked on the host before any GPU work, so this runs without a GPU too."""
    from custom_rasterizer_cuda import _lib

    L = _lib.lib
    rc = L.gs_rasterize_noalloc(1_000_000, 1080, 1920, 1, 1, 1, 1, 1, 8_000_000, 1, 1, 1, 1, 1,
                                None, None)
    assert rc == _lib.GS_ERR_CAPACITY
    msg = L.gs_last_error().decode()
    assert "fixed scratch holds 16777216 bytes" in msg and "gs_rasterize" in msg
