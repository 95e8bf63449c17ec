"""The C ABI library: it loads without a GPU, exports every entry point declared in
include/gs3d_b200.h, sizes workspaces on the host and rejects bad arguments before any CUDA
call (mirroring the reference's TORCH_CHECK errors as status codes)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "gs3d_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^GS_API\s+[\w\s\*]+?\b(gs_\w+)\s*\(", text, flags=re.M)


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("gs_project", "gs_sh_forward", "gs_rasterize", "gs_rasterize_backward",
                     "gs_sh_backward", "gs_project_backward", "gs_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from custom_rasterizer_cuda import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"symbols declared but not exported: {missing}"
    # the ctypes binding covers exactly the declared surface
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_version_and_no_error_initially():
    from custom_rasterizer_cuda import _lib

    assert b"sm_100a" in _lib.lib.gs_version()
    assert _lib.lib.gs_last_error() == b""


def test_workspace_size_is_host_only_and_monotone():
    from custom_rasterizer_cuda import _lib

    L = _lib.lib
    small = L.gs_rasterize_workspace_size(4096, 128, 128, 10_000)
    big = L.gs_rasterize_workspace_size(1_000_000, 1080, 1920, 8_000_000)
    assert 0 < small < big
    assert L.gs_rasterize_workspace_size(4096, 128, 128, 20_000) > small
    assert L.gs_rasterize_workspace_size(-1, 128, 128, 10) == 0
    assert L.gs_rasterize_backward_workspace_size(1000) >= 1000 * 48


@pytest.mark.parametrize("call", [
    lambda L: L.gs_project(-1, None, None, None, None, None, 1.0, 1.0, 0.0, 0.0, None, None,
                           None, None),
    lambda L: L.gs_sh_forward(-5, None, None, None, None, None, None),
    lambda L: L.gs_rasterize(4, 0, 16, None, None, None, None, None, None, 0, 0, None, None,
                             None, None, None, None, None, None, None),
    lambda L: L.gs_rasterize(4, 16, 16, None, None, None, None, None, None, 0, 0, None, None,
                             None, None, None, None, None, None, None),
    lambda L: L.gs_rasterize_backward(4, 16, 16, None, None, None, None, None, None, None,
                                      None, None, None, 0, None, None, None, None, None),
])
def test_invalid_arguments_rejected_before_cuda(call):
    from custom_rasterizer_cuda import _lib

    status = call(_lib.lib)
    assert status == _lib.GS_ERR_INVALID_ARG
    assert _lib.lib.gs_last_error() != b""


def test_zero_sized_calls_are_noops():
    from custom_rasterizer_cuda import _lib

    L = _lib.lib
    assert L.gs_project(0, None, None, None, None, None, 1.0, 1.0, 0.0, 0.0, None, None, None,
                        None) == 0
    assert L.gs_sh_forward(0, None, None, None, None, None, None) == 0
    assert L.gs_sh_backward(0, None, None, None, None, None, None, None, None, None) == 0


def test_python_boundary_checks_match_reference_messages():
    import torch
    import custom_rasterizer_cuda as crc

    cpu = torch.zeros(4, 3)
    with pytest.raises(RuntimeError, match="mu3d must be a CUDA tensor"):
        crc.project(4, cpu, torch.zeros(4, 4), torch.zeros(4, 3), torch.eye(3), torch.zeros(3),
                    1.0, 1.0, 0.0, 0.0)
    with pytest.raises(RuntimeError, match="camera_position must be a CUDA tensor"):
        crc.SH(4, torch.zeros(3), cpu, cpu, torch.zeros(4, 15, 3))
    # N == 0 returns the reference's empty buffers before any check (rasterize.cu:306-319)
    img, ids, ranges, final_T, n_contrib = crc.rasterize(0, cpu, cpu, cpu, cpu, cpu, 20, 40)
    assert img.shape == (20, 40, 3) and float(img.abs().sum()) == 0.0
    assert ids.numel() == 0 and ranges.shape == (2 * 3, 2)
    assert bool((final_T == 1).all()) and int(n_contrib.abs().sum()) == 0


def test_training_entry_points_reject_bad_arguments_before_cuda():
    """gs_adam_step, gs_sharded_adam_step, gs_render_forward and gs_render_backward validate
    on the host."""
    from custom_rasterizer_cuda import _lib

    L = _lib.lib
    sizes = (ctypes.c_longlong * 1)(8)
    lrs = (ctypes.c_float * 1)(1e-3)
    ptrs = (ctypes.c_void_p * 1)(16)
    # more than 8 groups, a zero step, a beta outside [0, 1)
    assert L.gs_adam_step(9, ptrs, sizes, lrs, 16, 16, 16, 0.9, 0.999, 1e-15, 1, None, None, None) == \
        _lib.GS_ERR_INVALID_ARG
    assert L.gs_adam_step(1, ptrs, sizes, lrs, 16, 16, 16, 0.9, 0.999, 1e-15, 0, None, None, None) == \
        _lib.GS_ERR_INVALID_ARG
    assert L.gs_adam_step(1, ptrs, sizes, lrs, 16, 16, 16, 1.0, 0.999, 1e-15, 1, None, None, None) == \
        _lib.GS_ERR_INVALID_ARG
    assert L.gs_adam_step(0, None, None, None, None, None, None, 0.9, 0.999, 1e-15, 1, None,
                          None, None) == 0

    import sys

    sys.path.insert(0, str(ROOT / "custom-3dgs-cuda_b200"))
    from gs3d_b200.sharded import ShardBuffers

    assert L.gs_sharded_adam_step(None, None, None, 1, sizes, lrs, 0.9, 0.999, 1e-15, 1, 1.0,
                                  None, None, None) == _lib.GS_ERR_INVALID_ARG
    d = ShardBuffers(world=2, rank=2, shard=8)  # rank out of range
    assert L.gs_sharded_adam_step(ctypes.addressof(d), 16, 16, 1, sizes, lrs, 0.9, 0.999, 1e-15,
                                  1, 1.0, None, None, None) == _lib.GS_ERR_INVALID_ARG
    assert b"rank" in L.gs_last_error()
    d = ShardBuffers(world=2, rank=0, shard=6)  # shard not a multiple of 4
    assert L.gs_sharded_adam_step(ctypes.addressof(d), 16, 16, 1, sizes, lrs, 0.9, 0.999, 1e-15,
                                  1, 1.0, None, None, None) == _lib.GS_ERR_INVALID_ARG
    # a clamp whose lower bound is above its upper bound
    lo, hi = (ctypes.c_float * 1)(1.0), (ctypes.c_float * 1)(0.0)
    assert L.gs_adam_step(1, ptrs, sizes, lrs, 16, 16, 16, 0.9, 0.999, 1e-15, 1, lo, hi,
                          None) == _lib.GS_ERR_INVALID_ARG
    assert b"clamp" in L.gs_last_error()
    # unknown render flag
    assert L.gs_render_forward(1, 16, 16, *([16] * 9), 1.0, 1.0, 8.0, 8.0, 256, 1 << 20, 16,
                               *([256] * 6), None, None, 0x80, None) == _lib.GS_ERR_INVALID_ARG
    assert b"flag" in L.gs_last_error()
    # the backward takes GS_RENDER_CONCURRENT only
    assert L.gs_render_backward(1, 16, 16, *([16] * 9), 1.0, 1.0, 8.0, 8.0, 256, 1 << 20,
                                *([256] * 4), 256, 1 << 20, *([256] * 7), 0, None, None, None,
                                1.0, 1.0, None, None, 1, None) == _lib.GS_ERR_INVALID_ARG
    assert b"flag" in L.gs_last_error()


def test_pair_capacity_memory_uses_the_last_count():
    """The pair-buffer guess for a (N, H, W, binning mode) is the last pair count seen + 12.5%
    + 4096, and counts of one binning mode do not leak into the other."""
    from custom_rasterizer_cuda import _capacity

    _capacity.update(123, 45, 67, 10_000, 1)
    assert _capacity.guess(123, 45, 67, 1) == 10_000 + 10_000 // 8 + 4096
    assert _capacity.guess(123, 45, 67, 0) == 8 * 123 + 4096
