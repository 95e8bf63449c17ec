"""The multi-GPU optimizer step: gradient reduce-scatter, Adam on each rank's shard and
parameter all-gather in one `gs_sharded_adam_step` kernel per rank.

The parameters, the gradient bucket and the max-statistic buffer live in symmetric memory
(torch.distributed._symmetric_memory, CUDA backend): the same layout on every rank, mapped into
every peer and, on NVSwitch systems, into one NVLink multicast range. Rank r owns a contiguous
1/world shard of the bucket and of the parameters and keeps the Adam moments of that shard only.
The kernel sums the shard over all ranks (multimem.ld_reduce in the switch, or peer loads),
applies Adam with gradient scale 1 / batch, and writes the new parameters and the reduced
densification statistics to every rank (multimem.st, or peer stores). This replaces an NCCL
all-reduce of the whole bucket followed by a full-size Adam on every rank.

`shard_layout` is the pure host-side layout (tested on CPU); `ShardedStep` needs CUDA GPUs, one
process per GPU, and an initialised process group.
"""

from __future__ import annotations

import ctypes
import math
import os
from ctypes import c_int, c_longlong, c_void_p
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .clamps import clamp_arrays


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass(frozen=True)
class ShardLayout:
    n_param: int        # parameter elements: gradients at [0, n_param) of the bucket
    stats_offset: int   # norm sums at [stats_offset, +N), counts at [stats_offset + N, +N)
    n_stats: int
    shard: int          # elements per rank (multiple of 4)
    length: int         # bucket / parameter buffer length = shard * world
    max_shard: int      # elements per rank of the max statistic
    max_length: int


def shard_layout(n_param: int, n_gaussians: int, world: int) -> ShardLayout:
    stats_offset = _round_up(n_param, 4)
    n_stats = 2 * n_gaussians
    shard = _round_up(max(1, math.ceil((stats_offset + n_stats) / world)), 4)
    max_shard = max(1, math.ceil(n_gaussians / world))
    return ShardLayout(n_param, stats_offset, n_stats, shard, shard * world, max_shard,
                       max_shard * world)


class ShardBuffers(ctypes.Structure):
    """Mirror of gs_shard_buffers (include/gs3d_b200.h)."""

    _fields_ = [("world", c_int), ("rank", c_int), ("shard", c_longlong),
                ("n_param", c_longlong), ("stats_offset", c_longlong), ("n_stats", c_longlong),
                ("max_shard", c_longlong), ("n_max", c_longlong),
                ("bucket", c_void_p), ("bucket_mc", c_void_p), ("bucket_peers", c_void_p),
                ("params", c_void_p), ("params_mc", c_void_p), ("params_peers", c_void_p),
                ("maxbuf", c_void_p), ("max_mc", c_void_p), ("max_peers", c_void_p),
                ("signal_pads", c_void_p), ("signal_slots", c_longlong),
                ("phase_ns", c_void_p), ("wait_ns", ctypes.c_ulonglong)]


class ShardedStep:
    """Symmetric parameter / gradient / statistic buffers of one rank and the sharded Adam.

    `param_views` are views of the parameter buffer in the shapes of `param_init`;
    `bucket` holds the gradients (first n_param elements, in parameter order) and the summed
    densification statistics; `max_stat` the per-Gaussian max statistic. `step()` runs the
    fused reduction + Adam + broadcast; afterwards every rank holds the same parameters and the
    reduced statistics, while each rank's gradient slice keeps its own (unreduced) sums.
    Two ranks use peer loads and stores, more ranks the NVLink multicast path where the
    machine has it; GS3D_SHARD_PEER=1 forces the peer path and =0 multicast.
    """

    def __init__(self, param_init: list[torch.Tensor], names: list[str], lrs: list[float],
                 n_gaussians: int, batch: int, device: torch.device, group=None,
                 betas=(0.9, 0.999), eps: float = 1e-15):
        import torch.distributed._symmetric_memory as symm

        from custom_rasterizer_cuda import _lib

        self._lib = _lib
        group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if len(param_init) > 8:
            raise ValueError("at most 8 parameter groups")
        sizes = [t.numel() for t in param_init]
        lay = shard_layout(sum(sizes), n_gaussians, self.world)
        self.layout = lay
        try:
            symm.set_backend("CUDA")
        except Exception:  # the backend is already fixed for this process
            pass
        f32 = torch.float32
        self.bucket = symm.empty(lay.length, dtype=f32, device=device)
        self.params = symm.empty(lay.length, dtype=f32, device=device)
        self.max_stat_buf = symm.empty(lay.max_length, dtype=f32, device=device)
        self.bucket.zero_()
        self.params.zero_()
        self.max_stat_buf.zero_()
        self.param_views = []
        off = 0
        for t, k in zip(param_init, sizes):
            v = self.params[off:off + k].view(t.shape)
            v.copy_(t.to(device=device, dtype=f32))
            self.param_views.append(v)
            off += k
        self.max_stat = self.max_stat_buf[:n_gaussians]
        self.exp_avg = torch.zeros(lay.shard, device=device, dtype=f32)
        self.exp_avg_sq = torch.zeros(lay.shard, device=device, dtype=f32)
        self.h_bucket = symm.rendezvous(self.bucket, group)
        self.h_params = symm.rendezvous(self.params, group)
        self.h_max = symm.rendezvous(self.max_stat_buf, group)
        for h in (self.h_bucket, self.h_params, self.h_max):
            off = getattr(h, "offset", 0)
            if (off() if callable(off) else off) != 0:
                # the kernel indexes from the multicast / peer buffer bases
                raise RuntimeError("symmetric tensor does not start at its buffer base")
        pad = self.h_bucket.get_signal_pad(self.rank)
        pad.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group)
        from torch._C._autograd import DeviceType
        from torch._C._distributed_c10d import _SymmetricMemory

        idx = device.index if device.index is not None else torch.cuda.current_device()
        # data path: peer loads / stores for two ranks (measured faster there: 0.54 vs 0.66 ms
        # per step on 2 B200s), NVLink multicast above; GS3D_SHARD_PEER=1 / 0 forces one
        forced = os.environ.get("GS3D_SHARD_PEER")
        want_mc = (forced == "0") if forced in ("0", "1") else self.world > 2
        use_mc = (want_mc and _SymmetricMemory.has_multicast_support(DeviceType.CUDA, idx)
                  and all(h.multicast_ptr != 0 for h in
                          (self.h_bucket, self.h_params, self.h_max)))
        self.multicast = use_mc
        self.desc = ShardBuffers(
            world=self.world, rank=self.rank, shard=lay.shard, n_param=lay.n_param,
            stats_offset=lay.stats_offset, n_stats=lay.n_stats, max_shard=lay.max_shard,
            n_max=n_gaussians,
            bucket=self.bucket.data_ptr(),
            bucket_mc=self.h_bucket.multicast_ptr if use_mc else None,
            bucket_peers=self.h_bucket.buffer_ptrs_dev,
            params=self.params.data_ptr(),
            params_mc=self.h_params.multicast_ptr if use_mc else None,
            params_peers=self.h_params.buffer_ptrs_dev,
            maxbuf=self.max_stat_buf.data_ptr(),
            max_mc=self.h_max.multicast_ptr if use_mc else None,
            max_peers=self.h_max.buffer_ptrs_dev,
            signal_pads=self.h_bucket.signal_pad_ptrs_dev,
            signal_slots=pad.numel() * pad.element_size() // 4)
        self.param_groups = [{"params": [v], "lr": float(lr), "name": n}
                             for v, lr, n in zip(self.param_views, lrs, names)]
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        self.batch = int(batch)
        self.n_steps = 0
        self._sizes = (c_longlong * len(sizes))(*sizes)
        self.device = device

    @property
    def grads(self) -> torch.Tensor:
        return self.bucket[:self.layout.n_param]

    def norm_sum(self, n: int) -> torch.Tensor:
        o = self.layout.stats_offset
        return self.bucket[o:o + n]

    def count(self, n: int) -> torch.Tensor:
        o = self.layout.stats_offset + n
        return self.bucket[o:o + n]

    def record_phases(self, steps: int) -> None:
        """Record the kernel phases (kernel start, end of the opening barrier, of the data loop,
        of the closing barrier; globaltimer ns) of the next `steps` steps; 0 turns it off. The
        rows are allocated and initialised here, so recording adds no host-device copy."""
        self.desc.phase_ns = None
        self._phase_rows = None
        self._phase_used = 0
        if steps > 0:
            init = torch.tensor([-1, 0, 0, 0], dtype=torch.int64)
            self._phase_rows = init.repeat(steps, 1).to(self.device)

    def phase_ms(self) -> dict | None:
        """Mean per-step phase durations (ms) of the recorded steps."""
        if self._phase_rows is None or self._phase_used == 0:
            return None
        p = self._phase_rows[:self._phase_used].cpu().to(torch.float64)
        d = (p[:, 1:] - p[:, :-1]) * 1e-6
        return {"opening_barrier": float(d[:, 0].mean()), "data": float(d[:, 1].mean()),
                "closing_barrier": float(d[:, 2].mean())}

    def step(self) -> None:
        rows = getattr(self, "_phase_rows", None)
        if rows is not None and self._phase_used < rows.shape[0]:
            self.desc.phase_ns = rows[self._phase_used].data_ptr()
            self._phase_used += 1
        else:
            self.desc.phase_ns = None
        self.n_steps += 1
        k = len(self.param_groups)
        lrs = (ctypes.c_float * k)(*[g["lr"] for g in self.param_groups])
        with torch.cuda.device(self.device):
            self._lib.check(self._lib.lib.gs_sharded_adam_step(
                ctypes.addressof(self.desc), self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(),
                k, self._sizes, lrs, self.betas[0], self.betas[1], self.eps, self.n_steps,
                1.0 / self.batch, *clamp_arrays(self.param_groups),
                torch.cuda.current_stream(self.device).cuda_stream))

    def zero_grad(self, set_to_none: bool = False) -> None:
        self.bucket.zero_()
        self.max_stat.zero_()
