"""The bounded wait of the multi-GPU optimizer kernel (gs_sharded_adam_step) runs out and is
reported, on one GPU and without a fault.

A two-rank step is emulated on one device: rank 0's kernel gets two signal pads and two copies
of the bucket and parameters, all in its own memory, and no second kernel ever arrives at the
barrier. With a 20 ms wait limit (gs_shard_buffers.wait_ns) every CTA's barrier wait gives up,
the kernel sets device error bit 8 and returns before touching any data, and the context stays
usable for the next call."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

PEER_TIMEOUT_BIT = 8


def test_sharded_step_barrier_wait_runs_out_and_is_reported(crc, cuda_device):
    from custom_rasterizer_cuda import _lib
    from gs3d_b200.sharded import ShardBuffers

    dev = cuda_device
    crc.clear_device_errors()
    world, shard = 2, 1024
    n_param = shard * world
    g = torch.Generator("cpu").manual_seed(3)
    bucket = [torch.rand(n_param, generator=g).to(dev) for _ in range(world)]
    params = [torch.rand(n_param, generator=g).to(dev) for _ in range(world)]
    before = [p.clone() for p in params]
    exp_avg = torch.zeros(shard, device=dev)
    exp_avg_sq = torch.zeros(shard, device=dev)
    slots = 4096
    pads = torch.zeros(world, slots, dtype=torch.int32, device=dev)

    def ptrs(ts):
        return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)

    pad_ptrs, bucket_ptrs, param_ptrs = ptrs(list(pads)), ptrs(bucket), ptrs(params)
    desc = ShardBuffers(
        world=world, rank=0, shard=shard, n_param=n_param, stats_offset=n_param, n_stats=0,
        max_shard=0, n_max=0, bucket=bucket[0].data_ptr(), bucket_mc=None,
        bucket_peers=bucket_ptrs.data_ptr(), params=params[0].data_ptr(), params_mc=None,
        params_peers=param_ptrs.data_ptr(), maxbuf=None, max_mc=None, max_peers=None,
        signal_pads=pad_ptrs.data_ptr(), signal_slots=slots, phase_ns=None,
        wait_ns=20_000_000)
    sizes = (ctypes.c_longlong * 1)(n_param)
    lrs = (ctypes.c_float * 1)(1e-3)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    _lib.check(_lib.lib.gs_sharded_adam_step(
        ctypes.addressof(desc), exp_avg.data_ptr(), exp_avg_sq.data_ptr(), 1, sizes, lrs, 0.9,
        0.999, 1e-15, 1, 1.0, None, None, torch.cuda.current_stream(dev).cuda_stream))
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    bits = crc.device_error_bits()
    crc.clear_device_errors()
    assert bits & PEER_TIMEOUT_BIT, bits
    assert elapsed < 2.0, elapsed  # ended at its 20 ms limit, not the 5 s default
    for p, b in zip(params, before):
        assert torch.equal(p, b)  # returned before the data phase
    assert float(exp_avg.abs().sum()) == 0.0
    # the context is still usable
    z = torch.ones(8, device=dev).sum()
    assert float(z) == 8.0
    assert crc.device_error_bits() == 0
