"""Benchmark of the B200 rasterizer: the view-parallel training step of config 4.

One step = a batch of 8 views (1920x1080, fx = fy = 1500) of the 1M-Gaussian clustered
scene (config 2's distribution, SH degree 3): forward + backward of every view through
`gaussian_splatting.rasterizer.rasterize` (the drop-in wrapper over libgs3d_b200), the
0.8 L1 + 0.2 (1 - SSIM) loss, densification statistics, one all-reduce of the flat gradient
bucket across ranks and an Adam update. The 8 views are split across the N ranks (strong
scaling); `value` is whole-job views/s with the targets resident in HBM, `e2e` the same
with every step's targets copied from pinned host memory and its loss read back.

Also reported (rank 0): forward / backward ms and FPS of one config-2 view, the roofline of
the dominant kernel, the kernel launch count, SM clocks sampled during the timed region and
the CPU baseline (the CPU oracle on one view).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "custom-3dgs-cuda_b200"
for _p in (str(PKG), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "fwd+bwd ms & FPS, 1M Gaussians SH3 @1080p; train views/s at 1/2/4/8 B200"
UNIT = "views/s"
BATCH_VIEWS = 8
N_GAUSSIANS = 1_000_000
WORKLOAD = ("config4: 1M clustered Gaussians (config-2 distribution), SH degree 3, batch of 8 "
            "views 1920x1080 fx=fy=1500 on a radius-8 sphere, L1+SSIM loss, grad all-reduce, Adam")


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=float(d["hbm_gbs"]), sm_max_mhz=float(d.get("sm_max_mhz", 1965.0)),
                    source="measured")
    return dict(hbm_gbs=6650.0, sm_max_mhz=1965.0, source="fallback")


# ---- clocks sampled during the timed region ------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                smax = max(smax, float(f[1]))
            except ValueError:
                continue
            for name, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- distributed plumbing --------------------------------------------------------------------
def init_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()


# ---- per-view breakdown (rank 0) -------------------------------------------------------------
def per_view_breakdown(trainer, view: dict, reps: int = 5) -> dict:
    """Forward / backward ms of one view through the wrapper and per C-ABI call timings."""
    import custom_rasterizer_cuda as crc
    from gaussian_splatting.rasterizer.rasterize import rasterize

    g = trainer.gaussians
    dev = trainer.device
    fwd, bwd = [], []
    for i in range(reps + 2):
        for p in trainer.params:
            p.grad = None
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        img = rasterize(g, view)
        e1.record()
        img.sum().backward()
        e2.record()
        torch.cuda.synchronize()
        if i >= 2:
            fwd.append(e0.elapsed_time(e1))
            bwd.append(e1.elapsed_time(e2))
    trainer.fg.rebind(trainer.params)

    # per C-ABI call (events on the launching stream)
    with torch.no_grad():
        mu, q, s, al, A, kj = (p.detach() for p in trainer.params)
        R, t = view["R"], view["T"]
        H, W = view["height"], view["width"]
        op = torch.sigmoid(al).contiguous()
        cam = (-(R.T @ t)).contiguous()
        stages = {}
        times = {k: [] for k in ("project", "SH", "rasterize", "backwards_rasterization",
                                 "backwards_SH", "backwards_projection")}
        for i in range(reps + 1):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
            ev[0].record()
            mean2d, cov2d, depths = crc.project(mu.shape[0], mu, q, s, R, t, view["fx"],
                                                view["fy"], view["cx"], view["cy"])
            ev[1].record()
            colors = crc.SH(mu.shape[0], cam, mu, A, kj)
            ev[2].record()
            img, ids, ranges, fT, nc = crc.rasterize(mu.shape[0], depths, mean2d, cov2d, colors,
                                                     op, H, W)
            ev[3].record()
            gimg = torch.ones_like(img)
            ev3b = torch.cuda.Event(enable_timing=True)
            ev3b.record()
            gm, gc, gcol, ga = crc.backwards_rasterization(gimg, mean2d, cov2d, colors, op, ids,
                                                           ranges, fT, nc, mu.shape[0], H, W)
            ev[4].record()
            crc.backwards_SH(gcol, mu, A, kj, cam)
            ev[5].record()
            crc.backwards_projection(gm, gc, mu, q, s, R, t, view["fx"], view["fy"], view["cx"],
                                     view["cy"])
            ev[6].record()
            torch.cuda.synchronize()
            if i >= 1:
                times["project"].append(ev[0].elapsed_time(ev[1]))
                times["SH"].append(ev[1].elapsed_time(ev[2]))
                times["rasterize"].append(ev[2].elapsed_time(ev[3]))
                times["backwards_rasterization"].append(ev3b.elapsed_time(ev[4]))
                times["backwards_SH"].append(ev[4].elapsed_time(ev[5]))
                times["backwards_projection"].append(ev[5].elapsed_time(ev[6]))
        for k, v in times.items():
            stages[k] = statistics.median(v)
        M = int(ids.numel())
        n_contrib_sum = int(nc.sum().item())
        visible = int((depths > 0).sum().item())
    return {"fwd_ms": statistics.median(fwd), "bwd_ms": statistics.median(bwd),
            "fps": 1000.0 / statistics.median(fwd), "stages_ms": stages, "pairs": M,
            "visible": visible, "replayed_pairs": n_contrib_sum}


def roofline_entry(bd: dict, pk: dict, n: int) -> dict:
    """Roofline of the dominant stage of one view. Blend stages are FP32-issue bound (no
    dense contraction anywhere); the per-Gaussian stages are HBM bound."""
    st = bd["stages_ms"]
    name = max(st, key=st.get)
    ms = st[name]
    # algorithmic bytes per Gaussian / flops per evaluated (pixel, Gaussian) pair
    bytes_per_g = {"project": 64, "SH": 216, "backwards_SH": 420, "backwards_projection": 100}
    if name in bytes_per_g:
        achieved = bytes_per_g[name] * n / (ms * 1e-3) / 1e9
        return {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": None,
                "peak_source": pk["source"]}
    fp32_peak = 148 * 128 * 2 * pk["sm_max_mhz"] * 1e6 / 1e12  # TFLOP/s
    flops_per_pair = 40.0 if name == "backwards_rasterization" else 14.0
    achieved = flops_per_pair * bd["replayed_pairs"] / (ms * 1e-3) / 1e12
    return {"kernel": name, "bound": "fp32", "achieved": achieved, "peak": fp32_peak,
            "unit": "TFLOP/s", "frac": achieved / fp32_peak, "traffic": None,
            "peak_source": "derived: 148 SMs x 128 FP32 lanes x 2 x sm_max_mhz"}


# ---- CPU baseline (the oracle) ----------------------------------------------------------------
def cpu_baseline_sample(scene, view, target) -> dict:
    """One view's forward + backward on the host cores through the CPU oracle."""
    import numpy as np

    from oracle import oracle as O

    O.build()
    threads = O.max_threads()
    O.set_threads(threads)
    R, t = view.R.numpy(), view.T.numpy()
    op = torch.sigmoid(scene.alpha).numpy().reshape(-1)
    t0 = time.perf_counter()
    out = O.render(scene.mu.numpy(), scene.q.numpy(), scene.s.numpy(), op, scene.A.numpy(),
                   scene.k_j.numpy(), R, t, view.fx, view.fy, view.cx, view.cy, view.height,
                   view.width)
    gimg = np.sign(out["img"] - target.numpy()).astype(np.float32) / out["img"].size
    gm, gc, gcol, ga, _ = O.rasterize_backward(gimg, out["mean2d"], out["cov2d"], out["colors"],
                                               op, out["sorted_ids"], out["tile_ranges"],
                                               out["final_T"], out["n_contrib"], view.height,
                                               view.width)
    O.sh_backward(gcol, scene.mu.numpy(), scene.A.numpy(), scene.k_j.numpy(),
                  O.camera_position(R, t))
    O.project_backward(gm, gc, scene.mu.numpy(), scene.q.numpy(), scene.s.numpy(), R, t,
                       view.fx, view.fy, view.cx, view.cy)
    dt = time.perf_counter() - t0
    return {"value": 1.0 / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "seconds": dt,
            "sample": "one 1920x1080 view of the 1M-Gaussian config-4 batch: projection, SH, "
                      "binning + stable 64-bit sort, blend, blend/SH/projection backward "
                      "(L1 gradient; the SSIM term and Adam are not in the CPU sample)"}


# ---- main -------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    """Reference arm: the reference has no CPU implementation of the path, so its CPU
    restatement (oracle/) is timed on the host cores, one view per step."""
    if rank != 0:
        return
    from gs3d_b200 import scenes

    sc, targets = scenes.config4(0, n=N_GAUSSIANS, n_views=BATCH_VIEWS)
    for _ in range(args.warmup_ref):
        cpu_baseline_sample(sc, sc.views[0], targets[0])
    secs = []
    res = None
    for k in range(args.steps):
        res = cpu_baseline_sample(sc, sc.views[k % BATCH_VIEWS], targets[k % BATCH_VIEWS])
        secs.append(res["seconds"])
    total = sum(secs)
    value = args.steps / total
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample": "one view per step", "inputs": "host"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": res["cores"], "kind": "port",
                             "sample": res["sample"]},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--gaussians", type=int, default=N_GAUSSIANS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup_ref = min(args.warmup, 1)
    rank, world, local = init_dist(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
            barrier(world)
            return 0
        return run_ours(args, rank, world, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


def run_ours(args, rank, world, local) -> int:
    import custom_rasterizer_cuda as crc
    from gs3d_b200 import scenes
    from gs3d_b200.train_step import Trainer

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sc, targets = scenes.config4(0, n=args.gaussians, n_views=BATCH_VIEWS)
    trainer = Trainer(sc, sc.views, [t.to(dev) for t in targets], dev, rank, world)
    mine = trainer.plan.views()
    host_targets = {vi: targets[vi].pin_memory() for vi in mine}
    h2d_bytes = sum(host_targets[vi].numel() * 4 for vi in mine)

    for _ in range(args.warmup):
        trainer.step()
    torch.cuda.synchronize()

    # ---- timed region: targets resident in HBM ----
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    sampler.start()
    launches0 = crc.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        trainer.step()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    launches = crc.kernel_launches() - launches0
    clocks = sampler.stop()
    elapsed_ms = max_over_ranks(e0.elapsed_time(e1), world)
    total_launches = int(sum_over_ranks(float(launches), world))

    # ---- e2e: targets copied from pinned host memory each step, loss read back ----
    barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    dev_targets = list(trainer.targets)
    for _ in range(args.steps):
        for vi in mine:
            dev_targets[vi] = host_targets[vi].to(dev, non_blocking=True)
        loss = trainer.step(dev_targets)
        float(loss.item())
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), world)

    value = BATCH_VIEWS * args.steps / (elapsed_ms * 1e-3)
    e2e_value = BATCH_VIEWS * args.steps / (e2e_ms * 1e-3)

    breakdown = None
    if rank == 0:
        v2 = scenes.config2(0, n=args.gaussians).views[0].as_dict(dev)
        breakdown = per_view_breakdown(trainer, v2)
    barrier(world)
    if rank != 0:
        return 0
    pk = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "gaussians": args.gaussians, "batch_views": BATCH_VIEWS,
                   "resolution": "1920x1080", "parallelism": f"views sharded over {world} rank(s)",
                   "l2": "inputs larger than L2 (236 MB of parameters + 25 MB per target)"},
        "per_view_config2": breakdown,
        "gpu_launches": total_launches,
        "gpu_launches_per_rank": launches,
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d_bytes * world,
                "d2h_bytes_per_step": 4 * world},
        "roofline": roofline_entry(breakdown, pk, args.gaussians),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(sc, sc.views[0], targets[0])
        line["cpu_baseline"].pop("seconds", None)
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
