"""The multi-GPU training step (gs_sharded_adam_step through gs3d_b200.sharded): two ranks, one
GPU each, each rendering half of a 4-view batch, against the single-GPU trainer on the whole
batch. Both data paths are run: NVLink multicast (multimem reductions and broadcasts in the
switch) and plain peer loads / stores. Both trainers clamp the opacity logits and log-scales
after each update (in the fused kernels). Skipped on machines with fewer than two GPUs."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

STEPS = 2
# clamps after each update (the reference trainer's kind, tighter so that they bind)
CLAMPS = {"alpha": (-1.0, 1.0), "s": (None, -4.0)}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup():
    from gs3d_b200 import scenes

    sc = scenes.config2(7, n=60_000)
    views = [scenes.pinhole(tuple(float(x) for x in e), 480, 270, 375.0)
             for e in ((0.0, 0.0, 8.0), (5.0, 2.0, 6.0), (-6.0, -1.0, 5.0), (1.0, -7.0, 4.0))]
    g = torch.Generator("cpu").manual_seed(9)
    targets = [torch.rand(270, 480, 3, generator=g) for _ in views]
    return sc, views, targets


def _snapshot(tr):
    return ([p.detach().cpu().clone() for p in tr.params], tr.fg.grad_norm_sum.cpu().clone(),
            tr.fg.grad_count.cpu().clone(), tr.fg.max_grad.cpu().clone())


def _worker(rank: int, world: int, port: int, peer: bool, q) -> None:
    import sys

    sys.path[:0] = [os.path.join(os.path.dirname(__file__), "..", "custom-3dgs-cuda_b200")]
    import torch.distributed as dist

    os.environ["GS3D_SHARD_PEER"] = "1" if peer else "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from custom_rasterizer_cuda import _lib
        from gs3d_b200.train_step import Trainer

        sc, views, targets = _setup()
        tr = Trainer(sc, views, [t.to(dev) for t in targets], dev, rank, world,
                     param_clamps=CLAMPS)
        for _ in range(STEPS):
            tr.step()
        torch.cuda.synchronize(dev)
        q.put((rank, tr.sharded.multicast, _lib.device_error_bits(), _snapshot(tr)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _close(mine, ref, rtol, atol, frac=1e-3):
    d = np.abs(mine - ref)
    ok = d <= atol + rtol * np.abs(ref)
    return ok.mean() >= 1.0 - frac, float(d.max())


@pytest.mark.parametrize("peer", [False, True], ids=["multicast", "peer"])
def test_sharded_step_matches_single_gpu(peer):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from gs3d_b200.train_step import LEARNING_RATES, PARAM_NAMES, Trainer

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, peer, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, rest) for r, *rest in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        multicast, errors, _ = got[r]
        assert errors == 0
        if not peer and not multicast:
            pytest.skip("no NVLink multicast on this machine")
        assert multicast == (not peer)

    dev = torch.device("cuda", 0)
    sc, views, targets = _setup()
    ref_tr = Trainer(sc, views, [t.to(dev) for t in targets], dev, param_clamps=CLAMPS)
    init = [p.detach().cpu().clone() for p in ref_tr.params]
    for _ in range(STEPS):
        ref_tr.step()
    torch.cuda.synchronize(dev)
    ref = _snapshot(ref_tr)

    p0, p1 = got[0][2][0], got[1][2][0]
    for a, b in zip(p0, p1):  # one writer per element: the ranks hold identical parameters
        assert torch.equal(a, b)
    for name, mine, theirs, start in zip(PARAM_NAMES, p0, ref[0], init):
        if name in CLAMPS:
            lo, hi = CLAMPS[name]
            assert float(mine.max()) <= hi and (lo is None or float(mine.min()) >= lo), name
        d_mine = (mine - start).numpy().ravel()
        d_ref = (theirs - start).numpy().ravel()
        assert np.abs(d_ref).max() > 0, name
        # Adam steps are bounded by ~lr per step; summation order only moves them by rounding
        ok, worst = _close(d_mine, d_ref, rtol=1e-3, atol=1e-7)
        assert ok, (name, worst)
        assert worst <= 2.5 * STEPS * LEARNING_RATES[name], (name, worst)
    for k, what in ((1, "norm sum"), (2, "count"), (3, "max")):
        for r in range(2):
            np.testing.assert_allclose(got[r][2][k].numpy(), ref[k].numpy(), rtol=1e-5,
                                       atol=1e-6, err_msg=what)
