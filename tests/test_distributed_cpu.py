"""The view-parallel step's host logic on gloo CPU ranks (world size 2 and 3): view sharding,
the flat gradient bucket, the SUM / MAX reductions of gradients and densification statistics,
and a rank failure surfacing as an error on the other rank instead of a hang."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 30.0) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _reduce_worker(rank: int, world: int, port: int, batch: int, q) -> None:
    import sys

    sys.path[:0] = [os.path.join(os.path.dirname(__file__), "..", "custom-3dgs-cuda_b200")]
    from gs3d_b200.train_step import FlatGrads, ShardPlan, accumulate_view_stats, reduce_step

    _init(rank, world, port)
    try:
        N = 5
        params = [torch.zeros(N, 3, requires_grad=True), torch.zeros(N, 1, requires_grad=True)]
        fg = FlatGrads(params, N)
        fg.zero()
        views = ShardPlan(rank, world, batch).views()
        for vi in views:
            # per-view gradient of value (vi + 1) everywhere; mean-2D grad marks Gaussian vi % N
            for p in params:
                p.grad.add_(float(vi + 1))
            g2 = torch.zeros(N, 2)
            g2[vi % N] = torch.tensor([0.3 * (vi + 1), 0.4 * (vi + 1)])
            accumulate_view_stats(fg, g2, width=2, height=2)
        reduce_step(fg, batch, world)
        q.put((rank, views, [p.grad.clone() for p in params], fg.grad_norm_sum.clone(),
               fg.grad_count.clone(), fg.max_grad.clone()))
    finally:
        dist.destroy_process_group()


def _run_ranks(target, world, extra, attempts=3):
    """Spawns `world` ranks of `target(rank, world, port, *extra, queue)` and collects one
    queue item per rank; further attempts with a fresh port cover a port another process took
    between _free_port() and the rendezvous (a rank that fails there can also break the result
    queue's pipe)."""
    import queue as queue_mod

    ctx = mp.get_context("spawn")
    for attempt in range(attempts):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=target, args=(r, world, port, *extra, q))
                 for r in range(world)]
        for p in procs:
            p.start()
        try:
            results = [q.get(timeout=120) for _ in range(world)]
        except (queue_mod.Empty, OSError, EOFError):
            results = None
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        if results is not None and all(p.exitcode == 0 for p in procs):
            return results
    raise AssertionError("ranks did not complete")


@pytest.mark.parametrize("world", [2, 3])
def test_view_sharding_and_reductions(world):
    batch = 8
    results = _run_ranks(_reduce_worker, world, (batch,))
    # every view rendered exactly once across ranks
    all_views = sorted(v for _, views, *_ in results for v in views)
    assert all_views == list(range(batch))
    expected_grad = sum(range(1, batch + 1)) / batch
    norms = {vi: 0.5 * (vi + 1) for vi in range(batch)}  # |(0.3k, 0.4k) * (1, 1)| = 0.5k
    for _, _, grads, nsum, count, gmax in results:
        for g in grads:
            assert torch.allclose(g, torch.full_like(g, expected_grad))
        for i in range(5):
            mine = [vi for vi in range(batch) if vi % 5 == i]
            assert nsum[i].item() == pytest.approx(sum(norms[v] for v in mine))
            assert count[i].item() == len(mine)
            assert gmax[i].item() == pytest.approx(max(norms[v] for v in mine))
    # all ranks agree exactly
    ref = results[0]
    for other in results[1:]:
        for a, b in zip(ref[2], other[2]):
            assert torch.equal(a, b)


def _failing_worker(rank: int, world: int, port: int, q) -> None:
    _init(rank, world, port, timeout_s=5.0)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except RuntimeError as e:
        q.put((rank, f"error: {type(e).__name__}"))


def test_failed_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1].startswith("error")
    assert got[0].startswith("error"), "the surviving rank must see the failure, not hang"


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("n_gaussians", [1, 5, 60_001])
def test_shard_layout_covers_the_bucket(world, n_gaussians):
    """Each rank's shard is a multiple of 4 elements, the shards tile the padded bucket, and the
    statistics start 16-byte aligned after the gradients."""
    import sys

    sys.path[:0] = [os.path.join(os.path.dirname(__file__), "..", "custom-3dgs-cuda_b200")]
    from gs3d_b200.sharded import shard_layout

    n_param = 59 * n_gaussians
    lay = shard_layout(n_param, n_gaussians, world)
    assert lay.shard % 4 == 0 and lay.stats_offset % 4 == 0
    assert lay.stats_offset >= n_param and lay.stats_offset - n_param < 4
    assert lay.length == lay.shard * world >= lay.stats_offset + lay.n_stats
    assert lay.length - (lay.stats_offset + lay.n_stats) < 4 * world + 4
    assert lay.max_length == lay.max_shard * world >= n_gaussians
