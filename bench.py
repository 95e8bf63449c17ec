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
import math
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
class NvmlClockSampler:
    """SM clock and clock-event reasons of one GPU sampled every 5 ms through NVML (the data
    `nvidia-smi --query-gpu=clocks.sm,...` prints) on a host thread while the timed region runs;
    short regions (a few ms per step at 8 GPUs) still get tens of samples."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, index: int):
        import threading

        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(index).uuid)
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            self.samples.append(float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)))
            bits = get_reasons(self.handle)
            for name, const in self.REASONS:
                if bits & getattr(nv, const, 0):
                    self.reasons.add(name)
            self._stop.wait(0.005)

    def start(self) -> None:
        self._thread.start()
        while not self.samples:  # the first sample precedes the timed region's start
            time.sleep(0.001)

    def stop(self) -> dict | None:
        self._stop.set()
        self._thread.join(timeout=5)
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml"}


def clock_sampler(index: int):
    try:
        return NvmlClockSampler(index)
    except Exception:
        return ClockSampler(index)


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

        # NCCL writes its banner and debug lines to stdout; keep stdout for the one JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
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


# ---- per-stage timing ----------------------------------------------------------------------
STAGES = {  # name: (start mark, end mark) of gs_set_stage_events
    "preprocess": (0, 1), "depth_sort": (1, 2), "duplicate": (2, 3), "tile_sort": (3, 4),
    "tile_order": (4, 5), "blend_forward": (5, 6), "blend_backward": (7, 8),
    "gaussian_backward": (10, 9),
}
N_MARKS = 11


class StageTimer:
    """One set of timed library events per (step, view); installed before each view renders
    so every render of the timed region is timed on its own stream."""

    def __init__(self, n_sets: int):
        from custom_rasterizer_cuda import _lib

        self._lib = _lib
        self.sets = [[_lib.Event(timed=True) for _ in range(N_MARKS)] for _ in range(n_sets)]
        self.used = 0

    def install_next(self) -> None:
        self._lib.set_stage_events(self.sets[self.used])
        self.used += 1

    def remove(self) -> None:
        self._lib.set_stage_events(None)

    def stage_ms(self, combined_views: int = 0) -> dict:
        """Mean ms per view of each stage. With `combined_views` = V > 0 the per-Gaussian
        backward ran once per step over the step's V views, while the last view's events were
        installed: its time is taken from every V-th set and divided by V."""
        out = {}
        sets = self.sets[:self.used]
        for name, (a, b) in STAGES.items():
            if name == "gaussian_backward" and combined_views:
                vals = [ev[a].elapsed_ms(ev[b]) / combined_views
                        for ev in sets[combined_views - 1::combined_views]]
            else:
                vals = [ev[a].elapsed_ms(ev[b]) for ev in sets]
            out[name] = statistics.mean(vals) if vals else None
        return out


def per_view_breakdown(trainer, view: dict, reps: int = 5) -> dict:
    """Forward / backward ms of one view through RasterizeFunction (CUDA events around the
    autograd calls) and its pair statistics."""
    from gaussian_splatting.rasterizer.rasterize import rasterize

    g = trainer.gaussians
    fwd, bwd = [], []
    for i in range(reps + 2):
        for p in trainer.params:
            p.grad = None
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        img = rasterize(g, view)
        e1.record()
        img.backward(torch.ones_like(img))
        e2.record()
        torch.cuda.synchronize()
        if i >= 2:
            fwd.append(e0.elapsed_time(e1))
            bwd.append(e1.elapsed_time(e2))
    trainer.fg.rebind(trainer.params)
    return {"fwd_ms": statistics.median(fwd), "bwd_ms": statistics.median(bwd),
            "fps": 1000.0 / statistics.median(fwd)}


def render_table(dev, reps: int = 10, only=None) -> dict:
    """Forward / backward ms and FPS through the drop-in `rasterize` / RasterizeFunction (the
    reference's binning) on the other synthetic scenes: BASELINE configs 0-3 and the
    reference's own bench scene (scripts/bench.py:30-63, the scene of its published numbers).
    fwd/bwd ms are medians of CUDA-event-timed single calls; fps is back-to-back forwards (the
    host's per-call work overlapping the previous frame), for config 3 over its 32 cameras."""
    from gaussian_splatting.rasterizer.rasterize import rasterize
    from gaussian_splatting.scene.gaussian import gaussian
    from gs3d_b200 import scenes
    from gs3d_b200.train_step import PARAM_NAMES

    def gaussians_of(sc):
        g = gaussian(sc.N)
        for name, p in zip(PARAM_NAMES, sc.params()):
            setattr(g, name, p.to(dev).contiguous().requires_grad_(True))
        return g

    def timed(fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        r = fn()
        b.record()
        return r, (a, b)

    def fwd_bwd(g, view):
        work = scene_work(g, view)
        fw, bw = [], []
        for i in range(reps + 2):
            for name in PARAM_NAMES:
                getattr(g, name).grad = None
            img, ev_f = timed(lambda: rasterize(g, view))
            grad = torch.ones_like(img)
            _, ev_b = timed(lambda: img.backward(grad))
            torch.cuda.synchronize()
            if i >= 2:
                fw.append(ev_f[0].elapsed_time(ev_f[1]))
                bw.append(ev_b[0].elapsed_time(ev_b[1]))
        with torch.no_grad():
            for _ in range(2):
                rasterize(g, view)
            torch.cuda.synchronize()
            def frames():  # each image dropped as the next renders, as a render loop does
                for _ in range(reps):
                    rasterize(g, view)

            _, ev = timed(frames)
            torch.cuda.synchronize()
        res = {"fwd_ms": statistics.median(fw), "bwd_ms": statistics.median(bw),
               "fps": reps / (ev[0].elapsed_time(ev[1]) * 1e-3)}
        res.update(render_roofline(work, res["fwd_ms"], res["bwd_ms"], pk))
        return res

    pk = peaks()
    out = {}
    want = (lambda name: only is None or name in only)
    if want("config0"):
        c0 = scenes.config0(0)
        out["config0_4096_128x128"] = fwd_bwd(gaussians_of(c0), c0.views[0].as_dict(dev))
    if want("config1"):
        c1 = scenes.config1(0)
        g1 = gaussians_of(c1)
        out["config1_100k_1280x720"] = fwd_bwd(g1, c1.views[0].as_dict(dev))
        out["config1_100k_1920x1080"] = fwd_bwd(g1, c1.views[1].as_dict(dev))
        del g1
    if want("reference_bench"):
        for w, h in ((1280, 720), (1920, 1080)):
            rb = scenes.reference_bench_scene(width=w, height=h)
            out[f"reference_bench_scene_100k_{w}x{h}"] = fwd_bwd(gaussians_of(rb),
                                                                 rb.views[0].as_dict(dev))
    if want("config2"):
        c2 = scenes.config2(0)
        out["config2_1M_1920x1080"] = fwd_bwd(gaussians_of(c2), c2.views[0].as_dict(dev))
    if not want("config3"):
        return out
    c3 = scenes.config3(0)
    g3 = gaussians_of(c3)
    views3 = [v.as_dict(dev) for v in c3.views]
    with torch.no_grad():
        for v in views3[:2]:
            rasterize(g3, v)
        torch.cuda.synchronize()
        def sweep():
            for v in views3:
                rasterize(g3, v)

        _, ev = timed(sweep)
        torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1])
    work = [scene_work(g3, v) for v in views3[::8]]
    mean_work = {k: statistics.mean(w[k] for w in work) for k in work[0]}
    res = {"fps": len(views3) / (ms * 1e-3), "fwd_ms_per_frame": ms / len(views3)}
    res.update(render_roofline(mean_work, ms / len(views3), None, pk))
    out["config3_3M_3840x2160_32_cameras"] = res
    return out


def scene_work(g, view) -> dict:
    """Units of work of one render of `view` through the fused path with the reference's
    binning (what RasterizeFunction runs): N Gaussians, P pixels, T tiles, M pairs, the
    (pixel, Gaussian) pairs an exact front-to-back blend must test (sum of n_contrib: each
    pixel's list walked to its last contributor) and E_f as the reference's blend evaluates
    them (every pixel of a tile tests each record until the whole tile is done, checked once per
    256-record batch: sum over tiles of 256 * min(K_t, ceil((max_p n_contrib_p + 1) / 256) *
    256), K_t the tile's list length)."""
    from custom_rasterizer_cuda.render import render_forward

    with torch.no_grad():
        op = torch.sigmoid(g.alpha.detach()).reshape(-1).contiguous()
        R, t = view["R"], view["T"]
        cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
        _, _, st = render_forward(g.mu.detach(), g.q.detach(), g.s.detach(), op, g.A.detach(),
                                  g.k_j.detach(), R, t, cam, view["fx"], view["fy"], view["cx"],
                                  view["cy"], view["height"], view["width"])
        H, W = view["height"], view["width"]
        tx, ty = (W + 15) // 16, (H + 15) // 16
        nc = st.n_contrib
        pad = torch.zeros((ty * 16, tx * 16), dtype=nc.dtype, device=nc.device)
        pad[:H, :W] = nc
        tile_max = pad.view(ty, 16, tx, 16).amax(dim=(1, 3)).reshape(-1).to(torch.int64)
        ranges = st.tile_ranges.to(torch.int64)
        K = ranges[:, 1] - ranges[:, 0]
        reach = torch.div(tile_max + 1 + 255, 256, rounding_mode="floor") * 256
        e_f = int((256 * torch.minimum(K, reach)).sum())
        return {"N": int(g.mu.shape[0]), "P": H * W, "T": tx * ty, "M": int(st.pairs),
                "sum_n_contrib": int(nc.to(torch.int64).sum()), "E_f": e_f}


# Algorithmic bytes of the HBM-bound stages of one fused render (RasterizeFunction), per unit:
# forward: parameters in (236 B/G) + blend record, rect and depth key out (48 + 8 + 8 B/G), the
# depth sort's four passes over 16 B/G, duplication (12 B/G in, 8 B per pair out), the tile
# sort's passes over 16 B per pair, the ranges (8 B per pair) and the image, transmittance and
# contributor count out (20 B per pixel); backward: the upstream image gradient, transmittance
# and counts in (20 B per pixel), then parameters, records and blend sums in (236 + 48 + 40
# B/G) and gradients out (236 B/G). FP32 work of the blends per tested pair: 14 flops forward,
# 40 flops backward.
def render_roofline(work: dict, fwd_ms: float, bwd_ms: float | None, pk: dict) -> dict:
    N, M, P, T = work["N"], work["M"], work["P"], work["T"]
    tile_passes = max(1, math.ceil(math.log2(max(T, 2)) / 8))
    fwd_bytes = (236 + 64) * N + 4 * 16 * N + 12 * N + 8 * M + tile_passes * 16 * M + 8 * M + 20 * P
    bwd_bytes = 20 * P + (236 + 48 + 40 + 236) * N
    fp32 = 148 * 128 * 2 * pk["sm_max_mhz"] * 1e6
    hbm = pk["hbm_gbs"] * 1e9
    fwd_floor = fwd_bytes / hbm + 14.0 * work["sum_n_contrib"] / fp32
    out = {"work": work, "fwd_roofline_ms": 1e3 * fwd_floor,
           "fwd_roofline_frac": 1e3 * fwd_floor / fwd_ms}
    if bwd_ms is not None:
        bwd_floor = bwd_bytes / hbm + 40.0 * work["sum_n_contrib"] / fp32
        out.update({"bwd_roofline_ms": 1e3 * bwd_floor, "bwd_roofline_frac": 1e3 * bwd_floor / bwd_ms})
    out["roofline_model"] = ("HBM-bound stages at their algorithmic bytes / measured HBM peak plus "
                             "the blends' FP32 work (sum of n_contrib tested pairs) / derived FP32 "
                             "peak, serialised; frac = that floor / the measured time")
    return out


def six_op_times(mod, dev, reps: int = 7) -> dict:
    """CUDA-event medians (ms) of the reference API's six ops, chained as its wrapper chains
    them, on config 2 (1M clustered Gaussians, 1920x1080) through module `mod` (this library's
    custom_rasterizer_cuda, or the reference's own extension)."""
    from gs3d_b200 import scenes

    sc = scenes.config2(0)
    view = sc.views[0]
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    R, t = view.R.to(dev).contiguous(), view.T.to(dev).contiguous()
    cam = (-(R.T @ t)).contiguous()
    op = torch.sigmoid(al).contiguous()
    H, W = view.height, view.width
    g = torch.rand(H, W, 3, generator=torch.Generator().manual_seed(5)).to(dev)
    names = ("project", "SH", "rasterize", "backwards_rasterization", "backwards_SH",
             "backwards_projection")
    times = {k: [] for k in names}
    for k in range(reps + 2):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        ev[0].record()
        m2, c2, d = mod.project(sc.N, mu, q, s, R, t, view.fx, view.fy, view.cx, view.cy)
        ev[1].record()
        col = mod.SH(sc.N, cam, mu, A, kj)
        ev[2].record()
        img, ids, ranges, fT, nc = mod.rasterize(sc.N, d, m2, c2, col, op, H, W)
        ev[3].record()
        gm, gc, gcol, ga = mod.backwards_rasterization(g, m2, c2, col, op, ids, ranges, fT, nc,
                                                       sc.N, H, W)
        ev[4].record()
        mod.backwards_SH(gcol, mu, A, kj, cam)
        ev[5].record()
        mod.backwards_projection(gm, gc, mu, q, s, R, t, view.fx, view.fy, view.cx, view.cy)
        ev[6].record()
        torch.cuda.synchronize()
        if k >= 2:
            for i, name in enumerate(names):
                times[name].append(ev[i].elapsed_time(ev[i + 1]))
    out = {k: statistics.median(v) for k, v in times.items()}
    out["fwd_ms"] = out["project"] + out["SH"] + out["rasterize"]
    out["bwd_ms"] = out["backwards_rasterization"] + out["backwards_SH"] + out["backwards_projection"]
    out["workload"] = "config2: 1M clustered Gaussians, 1920x1080, the six ops chained"
    return out


def reference_extension_b200(dev) -> dict:
    """The reference's own CUDA extension (all six ops: csrc/bindings.cpp built unmodified by
    oracle/build_ref.py, projection/SH against the GLM stand-in, "ref+shim") timed on this
    GPU at config 2, as north_star asks beside every number."""
    path = str(ROOT / "oracle" / "_ref" / "ref_full")
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import ref_full
    except ImportError as e:
        return {"unavailable": f"reference extension not built (oracle/build_ref.py): {e}"}
    out = six_op_times(ref_full, dev)
    out["build"] = ("ref+shim: the reference's bindings.cpp and six .cu files unmodified, sm_100a, "
                    "GLM API stand-in oracle/glm_shim")
    return out


def view_pair_stats(trainer, views: list[dict]) -> dict:
    """Pairs M and replayed (pixel, Gaussian) pairs (sum of n_contrib) of each view, with the
    binning the trainer uses (with tight bins both count only the shorter lists' entries)."""
    from custom_rasterizer_cuda.render import render_forward

    pairs, replayed = [], []
    with torch.no_grad():
        mu, q, s, al, A, kj = (p.detach() for p in trainer.params)
        op = torch.sigmoid(al).contiguous()
        for v in views:
            R, t = v["R"], v["T"]
            cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
            _, _, st = render_forward(mu, q, s, op, A, kj, R, t, cam, v["fx"], v["fy"], v["cx"],
                                      v["cy"], v["height"], v["width"],
                                      tight_bins=getattr(trainer, "tight_bins", False))
            pairs.append(st.pairs)
            replayed.append(int(st.n_contrib.sum().item()))
    return {"pairs": pairs, "replayed_pairs": replayed}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of each stage's kernel,
# from one `ncu --clock-control none` capture per kernel (one launch each) of a config-2 view
# (1M Gaussians of the config-4 distribution at 1920x1080) with the training step's kernels:
# `bench.py --view-only --view-throughput --steps 1 --warmup 1` (profiles/config2_view_kernels.md).
NCU_DRAM_BYTES = {
    "preprocess": 285.4e6, "duplicate": 12.0e6, "blend_forward": 66.8e6,
    "blend_backward": 133.5e6, "gaussian_backward": 460.5e6,
}
# warp instructions (smsp__inst_executed.sum) per launch of the blend kernels from the same
# captures: the blends are bound by instruction issue (one warp instruction per cycle on each
# of the 4 x 148 schedulers), not by FP32 FMA throughput
NCU_WARP_INST = {"blend_forward": 289.7e6, "blend_backward": 550.5e6}


def roofline_entry(stage_ms: dict, stats: dict, n_views_timed: int, pk: dict, n: int,
                   combined_views: int = 0,
                   name: str | None = None) -> dict:
    """Roofline of one stage (default: the dominant one) over the timed region. The blends are
    FP32-issue bound (no dense contraction anywhere on the path); the per-Gaussian stages are
    HBM bound."""
    if name is None:
        name = max((k for k in stage_ms if stage_ms[k] is not None), key=lambda k: stage_ms[k])
    ms = stage_ms[name]
    mean_replayed = statistics.mean(stats["replayed_pairs"])
    mean_pairs = statistics.mean(stats["pairs"])
    # algorithmic bytes per launch: per-unit bytes of each kernel times the units it processes
    hbm_bytes = {
        "preprocess": 236 * n + 56 * n,             # parameters in; rects + records out
        "depth_sort": 4 * 16 * n,                   # 4 passes over (key, id) of N_v <= N
        "duplicate": 12 * n + 8 * mean_pairs,
        "tile_sort": 2 * 16 * mean_pairs,
        # per view: its blend sums in; parameters in, gradients out (read-modify-write after
        # the first view) and statistics, once per view, or once per step over V views
        "gaussian_backward": (48 * n + (232 * n + 236 * n + 24 * n) / combined_views
                              if combined_views else 48 * n + 236 * n + 236 * n + 8 * n),
    }
    if name in hbm_bytes:
        achieved = hbm_bytes[name] / (ms * 1e-3) / 1e9
        return {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                "traffic": NCU_DRAM_BYTES.get(name),
                "peak_source": pk["source"], "ms_per_launch": ms}
    fp32_peak = 148 * 128 * 2 * pk["sm_max_mhz"] * 1e6 / 1e12  # TFLOP/s
    flops_per_pair = 40.0 if name == "blend_backward" else 14.0
    achieved = flops_per_pair * mean_replayed / (ms * 1e-3) / 1e12
    entry = {"kernel": name, "bound": "fp32", "achieved": achieved, "peak": fp32_peak,
             "unit": "TFLOP/s", "frac": achieved / fp32_peak,
             "traffic": NCU_DRAM_BYTES.get(name), "traffic_unit": "bytes per launch (ncu)",
             "peak_source": "derived: 148 SMs x 128 FP32 lanes x 2 x sm_max_mhz",
             "ms_per_launch": ms,
             "unit_of_work": f"{flops_per_pair:.0f} FLOP per replayed (pixel, Gaussian) pair, "
                             f"{mean_replayed:.3g} per view"}
    if name in NCU_WARP_INST:
        issue_peak = 148 * 4 * pk["sm_max_mhz"] * 1e6 / 1e9  # G warp instructions/s
        issued = NCU_WARP_INST[name] / (ms * 1e-3) / 1e9
        entry["issue"] = {"achieved": issued, "peak": issue_peak, "unit": "G warp inst/s",
                          "frac": issued / issue_peak,
                          "warp_inst_per_launch": NCU_WARP_INST[name],
                          "source": "ncu smsp__inst_executed.sum of the same kernel variant"}
    return entry


# ---- CPU baseline (the oracle) ----------------------------------------------------------------
def cpu_baseline_sample(scene, view, target, adam_seconds: float | None = None) -> dict:
    """One view of the training step on the host cores: the CPU oracle's forward and backward
    (projection, SH, binning + stable sort, blend, blend / SH / projection backward) with the
    step's loss (0.8 L1 + 0.2 (1 - SSIM), its torch formulation on the CPU, whose autograd gives
    the image gradient) and one eighth of a CPU Adam step over all parameters (the step's
    optimizer work per view; `adam_seconds` from `cpu_adam_seconds`)."""
    import numpy as np

    from gs3d_b200.train_step import gaussian_window, reconstruction_loss
    from oracle import oracle as O

    O.build()
    threads = O.max_threads()
    O.set_threads(threads)
    torch.set_num_threads(threads)
    R, t = view.R.numpy(), view.T.numpy()
    op = torch.sigmoid(scene.alpha).numpy().reshape(-1)
    window = gaussian_window()
    t0 = time.perf_counter()
    out = O.render(scene.mu.numpy(), scene.q.numpy(), scene.s.numpy(), op, scene.A.numpy(),
                   scene.k_j.numpy(), R, t, view.fx, view.fy, view.cx, view.cy, view.height,
                   view.width)
    img = torch.from_numpy(out["img"]).requires_grad_(True)
    loss = reconstruction_loss(img, target, window)
    loss.backward()
    gimg = img.grad.numpy().astype(np.float32)
    gm, gc, gcol, ga, _ = O.rasterize_backward(gimg, out["mean2d"], out["cov2d"], out["colors"],
                                               op, out["sorted_ids"], out["tile_ranges"],
                                               out["final_T"], out["n_contrib"], view.height,
                                               view.width)
    O.sh_backward(gcol, scene.mu.numpy(), scene.A.numpy(), scene.k_j.numpy(),
                  O.camera_position(R, t))
    O.project_backward(gm, gc, scene.mu.numpy(), scene.q.numpy(), scene.s.numpy(), R, t,
                       view.fx, view.fy, view.cx, view.cy)
    dt = time.perf_counter() - t0
    if adam_seconds is not None:
        dt += adam_seconds / BATCH_VIEWS
    return {"value": 1.0 / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "seconds": dt,
            "sample": "one 1920x1080 view of the 1M-Gaussian config-4 batch: projection, SH, "
                      "binning + stable 64-bit sort, blend, the L1 + SSIM loss and its image "
                      "gradient, blend/SH/projection backward, and 1/8 of an Adam step over "
                      "all parameters (the step's optimizer work per view)"}


def torch_cpu_config0(table: dict | None) -> dict:
    """BASELINE config 0's step (4,096 Gaussians at 128x128: forward, then the backward of L1
    against a seeded target) by the vectorised PyTorch restatement on the host cores, beside the
    same step on the GPU through RasterizeFunction (the render table's config-0 row)."""
    from gs3d_b200 import scenes
    from oracle import torch_cpu

    torch.set_num_threads(os.cpu_count() or 1)
    sc = scenes.config0(0)
    view = sc.views[0]
    target = torch.rand(view.height, view.width, 3, generator=torch.Generator().manual_seed(1))
    seconds, threads = torch_cpu.step_seconds(sc, view, target)
    out = {"value": 1.0 / seconds, "unit": "config-0 steps/s", "cores": threads,
           "kind": "torch-cpu restatement (oracle/torch_cpu.py)",
           "sample": "config 0: 4,096 Gaussians, 128x128, forward + L1 backward, median of 3"}
    row = (table or {}).get("config0_4096_128x128")
    if row:
        gpu_ms = row["fwd_ms"] + row["bwd_ms"]
        out["gpu_same_step_ms"] = gpu_ms
        out["gpu_over_cpu"] = seconds * 1e3 / gpu_ms
    return out


def cpu_adam_seconds(scene) -> float:
    """Seconds of one torch.optim.Adam step (eps 1e-15, the step's learning rates) over all
    parameters on the host cores."""
    from gs3d_b200.train_step import LEARNING_RATES, PARAM_NAMES

    params = [p.detach().clone().requires_grad_(True) for p in scene.params()]
    for p in params:
        p.grad = torch.randn_like(p) * 1e-3
    opt = torch.optim.Adam([{"params": [p], "lr": LEARNING_RATES[n]}
                            for p, n in zip(params, PARAM_NAMES)], eps=1e-15)
    opt.step()  # state allocation outside the timing
    t0 = time.perf_counter()
    opt.step()
    return time.perf_counter() - t0


def bench_config(args, world: int) -> dict:
    """The workload both arms report (the reference arm times a bounded sample of it on the
    host cores; its `cpu_baseline.sample` says which)."""
    return {"workload": WORKLOAD, "gaussians": args.gaussians, "batch_views": BATCH_VIEWS,
            "resolution": "1920x1080", "parallelism": f"views sharded over {world} rank(s)",
            "l2": "inputs larger than L2 (236 MB of parameters + 25 MB per target)"}


# ---- main -------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    """Reference arm: the reference has no CPU implementation of the path, so its CPU
    restatement (oracle/) is timed on the host cores, one view per step."""
    if rank != 0:
        return
    from gs3d_b200 import scenes

    sc, targets = scenes.config4(0, n=args.gaussians, n_views=BATCH_VIEWS)
    adam_s = cpu_adam_seconds(sc)
    for _ in range(args.warmup_ref):
        cpu_baseline_sample(sc, sc.views[0], targets[0], adam_s)
    secs = []
    res = None
    for k in range(args.steps):
        res = cpu_baseline_sample(sc, sc.views[k % BATCH_VIEWS], targets[k % BATCH_VIEWS],
                                  adam_s)
        secs.append(res["seconds"])
    total = sum(secs)
    value = args.steps / total
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": bench_config(args, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": res["cores"], "kind": "port",
                             "sample": res["sample"]},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if torch.cuda.is_available():
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        line["reference_extension_b200"] = reference_extension_b200(dev)
    emit(line)


# Where the JSON line goes: the process's original stdout. main() points file descriptor 1 at
# stderr so that library banners (NCCL's version line, for one) cannot precede the line.
OUT = sys.stdout


def emit(line: dict) -> None:
    print(json.dumps(line), file=OUT, flush=True)


def main() -> int:
    global OUT
    sys.stdout.flush()
    OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--gaussians", type=int, default=N_GAUSSIANS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-render-table", action="store_true",
                    help="skip the per-scene forward/backward/FPS table (configs 1-3)")
    ap.add_argument("--view-streams", type=int, default=8,
                    help="CUDA streams the views of a step alternate over (1 = in order)")
    ap.add_argument("--view-only", action="store_true",
                    help="forward+backward of one config-2 view per step (single GPU); a small "
                         "fixed workload for profiler captures of single kernels")
    ap.add_argument("--view-throughput", action="store_true",
                    help="with --view-only: the training step's kernel variants (tight bins, "
                         "GS_RENDER_CONCURRENT blend kernels) instead of the single-view ones")
    ap.add_argument("--six-op", action="store_true",
                    help="the reference API's six ops on one config-2 view per step (single "
                         "GPU), through this library; a small fixed workload for profiler "
                         "captures of the six-op kernels")
    ap.add_argument("--table-only", action="store_true",
                    help="only the per-scene forward/backward/FPS table (single GPU)")
    ap.add_argument("--table-scenes", default=None,
                    help="comma list of config0,config1,reference_bench,config2,config3")
    args = ap.parse_args()
    if args.view_only:
        return run_view(args)
    if args.six_op:
        import custom_rasterizer_cuda as crc

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        emit({"mode": "six_op", "six_op_config2": six_op_times(crc, dev, reps=args.steps)})
        return 0
    if args.table_only:
        torch.cuda.set_device(0)
        only = set(args.table_scenes.split(",")) if args.table_scenes else None
        emit({"mode": "render_table",
              "render_table": render_table(torch.device("cuda", 0), only=only)})
        return 0
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


def run_view(args) -> int:
    """One config-2 view (1M Gaussians, 1920x1080) rendered forward and backward through the
    fused path per step, with a seeded upstream image gradient; prints per-stage ms."""
    from custom_rasterizer_cuda import _lib
    from custom_rasterizer_cuda.render import render_backward, render_forward
    from gs3d_b200 import scenes

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sc = scenes.config2(0, n=args.gaussians)
    v = sc.views[0].as_dict(dev)
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    op = torch.sigmoid(al).reshape(-1).contiguous()
    cam = (-torch.matmul(v["R"].T, v["T"])).reshape(3).contiguous()
    g = torch.Generator("cpu").manual_seed(5)
    grad_img = torch.rand(v["height"], v["width"], 3, generator=g).to(dev)
    timer = StageTimer(args.steps)
    for k in range(args.warmup + args.steps):
        if k >= args.warmup:
            timer.install_next()
        img, _, st = render_forward(mu, q, s, op, A, kj, v["R"], v["T"], cam, v["fx"], v["fy"],
                                    v["cx"], v["cy"], v["height"], v["width"],
                                    tight_bins=args.view_throughput,
                                    concurrent=args.view_throughput)
        render_backward(st, grad_img, mu, q, s, A, kj, v["R"], v["T"], cam, v["fx"], v["fy"],
                        v["cx"], v["cy"], want_mean2d_grad=False)
    torch.cuda.synchronize()
    timer.remove()
    if _lib.device_error_bits() != 0:
        raise RuntimeError(f"device error bits {_lib.device_error_bits():#x}")
    emit({"mode": "view", "workload": "config2 view 0: 1M Gaussians, 1920x1080",
          "kernels": ("training-step variants (tight bins, throughput blend kernels)"
                      if args.view_throughput else "reference binning, latency blend kernels"),
          "steps": args.steps, "warmup": args.warmup, "pairs": st.pairs,
          "stage_ms": timer.stage_ms()})
    return 0


def run_ours(args, rank, world, local) -> int:
    import custom_rasterizer_cuda as crc
    from gs3d_b200 import scenes
    from gs3d_b200.train_step import HostTargets, Trainer

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sc, targets = scenes.config4(0, n=args.gaussians, n_views=BATCH_VIEWS)
    trainer = Trainer(sc, sc.views, [t.to(dev) for t in targets], dev, rank, world,
                      view_streams=args.view_streams)
    mine = trainer.plan.views()
    host_targets = {vi: targets[vi].pin_memory() for vi in mine}
    h2d_bytes = sum(host_targets[vi].numel() * 4 for vi in mine)

    for _ in range(args.warmup):
        trainer.step()
    torch.cuda.synchronize()

    # ---- timed region: targets resident in HBM ----
    sampler = clock_sampler(local)
    # CUDA events around each step's optimizer update (gradient reduction across ranks + Adam)
    update_events = []
    plain_update = trainer._update

    def timed_update():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        plain_update()
        b.record()
        update_events.append((a, b))

    trainer._update = timed_update
    if trainer.sharded is not None:
        trainer.sharded.record_phases(args.steps)
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
    trainer._update = plain_update
    update_ms = statistics.mean(a.elapsed_time(b) for a, b in update_events)
    update_phases = None
    if trainer.sharded is not None:
        update_phases = trainer.sharded.phase_ms()
        trainer.sharded.record_phases(0)
    launches = crc.kernel_launches() - launches0
    clocks = sampler.stop()
    elapsed_ms = max_over_ranks(e0.elapsed_time(e1), world)

    # ---- per-stage library timings (untimed steps, views in order on one stream, so that each
    # stage's events bracket only its own kernels) ----
    stage_steps = min(args.steps, 5)
    timer = StageTimer(stage_steps * len(mine))
    for _ in range(stage_steps):
        trainer.step(before_view=lambda vi: timer.install_next())
    torch.cuda.synchronize()
    timer.remove()
    stage_ms = timer.stage_ms(len(mine) if trainer.combined_backward else 0)
    total_launches = int(sum_over_ranks(float(launches), world))

    # ---- e2e: every step copies its targets from pinned host memory (side stream, each view's
    # loss waits for its own copy) and reads its loss back to the host (one step behind, so the
    # host keeps the device fed); all of it inside the timed region ----
    staged = HostTargets(host_targets, dev)
    assert staged.bytes_per_step == h2d_bytes
    trainer.step(staged)  # untimed: first use of the copy stream
    loss_host = torch.empty(args.steps, dtype=torch.float32, pin_memory=True)
    read = [torch.cuda.Event() for _ in range(args.steps)]
    losses = []
    barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for k in range(args.steps):
        loss = trainer.step(staged)
        loss_host[k].copy_(loss, non_blocking=True)
        read[k].record()
        if k > 0:
            read[k - 1].synchronize()
            losses.append(float(loss_host[k - 1]))
    read[-1].synchronize()
    losses.append(float(loss_host[-1]))
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), world)
    assert len(losses) == args.steps and all(math.isfinite(x) for x in losses)

    value = BATCH_VIEWS * args.steps / (elapsed_ms * 1e-3)
    e2e_value = BATCH_VIEWS * args.steps / (e2e_ms * 1e-3)

    breakdown = None
    stats = view_pair_stats(trainer, [trainer.views[vi] for vi in mine])
    if rank == 0:
        v2 = scenes.config2(0, n=args.gaussians).views[0].as_dict(dev)
        breakdown = per_view_breakdown(trainer, v2)
        breakdown.update({f"{k}_pairs": v for k, v in view_pair_stats(trainer, [v2]).items()})
    barrier(world)
    if rank != 0:
        return 0
    pk = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": bench_config(args, world),
        "per_view_config2": breakdown,
        "stage_ms_per_view": stage_ms,
        "view_streams": len(trainer._streams) or 1,
        "tight_bins": trainer.tight_bins,
        "blend_variant": ("throughput: 2 / 4 pixels per thread forward / backward"
                          if trainer.concurrent_views else
                          "latency: 1 / 2 pixels per thread forward / backward"),
        "per_gaussian_backward": ("once per step over the rank's views"
                                  if trainer.combined_backward else "once per view"),
        "update_ms_per_step": update_ms,
        "update_phases_ms_rank0": update_phases,
        "update": ("fused reduce-scatter + sharded Adam + all-gather (multicast)"
                   if trainer.sharded is not None and trainer.sharded.multicast else
                   "fused reduce-scatter + sharded Adam + all-gather (peer memory)"
                   if trainer.sharded is not None else "single-launch Adam"),
        "views_pairs": stats,
        "gpu_launches": total_launches,
        "gpu_launches_per_rank": launches,
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d_bytes * world,
                "d2h_bytes_per_step": 4 * world},
        "roofline": roofline_entry(stage_ms, stats, args.steps * len(mine), pk, args.gaussians,
                                   len(mine) if trainer.combined_backward else 0),
        "roofline_blend_forward": roofline_entry(stage_ms, stats, args.steps * len(mine), pk,
                                                 args.gaussians, name="blend_forward"),
    }
    if world == 1:
        line["six_op_config2"] = six_op_times(crc, dev)
    if world == 1 and not args.no_render_table:
        line["render_table"] = render_table(dev)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(sc, sc.views[0], targets[0],
                                                   cpu_adam_seconds(sc))
        line["cpu_baseline"].pop("seconds", None)
        line["cpu_baseline_torch"] = torch_cpu_config0(line.get("render_table"))
    emit(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
