"""View-parallel training step (the benchmark's config 4).

A batch of B camera views is split across the ranks of a process group (rank r renders views
r, r + world, ...). Every rank holds the full Gaussian set and the Adam state. Per step each
rank renders its views with the drop-in rasterizer, backpropagates
0.8 * L1 + 0.2 * (1 - SSIM) per view, and accumulates parameter gradients into ONE flat fp32
bucket (the parameters' .grad tensors are views into it). One all-reduce (SUM) of the bucket
and a divide by B then give every rank the batch-mean gradient, and Adam runs on every rank
identically. The densification statistics of the reference trainer
(gaussian_splatting/utils/adc.py:58-87: the per-Gaussian sum and count of the screen-space
mean-gradient norm scaled by (W/2, H/2)) are SUM-reduced with the bucket; the per-Gaussian
maximum of that norm over the batch is MAX-reduced separately.

With world size 1 no collective runs. Collectives go through torch.distributed (NCCL on GPUs,
gloo in the CPU tests).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

PARAM_NAMES = ("mu", "q", "s", "alpha", "A", "k_j")
# Adam learning rates of config 4 (means, quaternions, log-scales, opacity, SH DC, SH rest)
LEARNING_RATES = {"mu": 1.6e-4, "q": 1e-3, "s": 5e-3, "alpha": 5e-2, "A": 2.5e-3, "k_j": 2.5e-3}
LAMBDA_DSSIM = 0.2


def gaussian_window(size: int = 11, sigma: float = 1.5, device=None,
                    dtype=torch.float32) -> torch.Tensor:
    x = torch.arange(size, dtype=dtype, device=device) - (size - 1) / 2.0
    g = torch.exp(-(x * x) / (2.0 * sigma * sigma))
    g = g / g.sum()
    return torch.outer(g, g)


def ssim(img: torch.Tensor, ref: torch.Tensor, window: torch.Tensor) -> torch.Tensor:
    """Mean SSIM of two [H, W, 3] images as the reference's loss computes it
    (gaussian_splatting/utils/loss.py:8-33, torchmetrics structural_similarity_index_measure
    with data_range=1.0): both images clamped to [0, 1], an 11x11 Gaussian window (sigma 1.5),
    C1 = 0.01^2, C2 = 0.03^2, variances clamped at 0, the map averaged over the channels and
    the (H-10) x (W-10) positions whose window lies inside the image. torchmetrics reflect-pads
    by 5 and crops 5 from each side of the map, which leaves exactly those positions, so the
    valid (unpadded) convolution below gives the same value."""
    x = img.permute(2, 0, 1).unsqueeze(0).clamp(0.0, 1.0)
    y = ref.permute(2, 0, 1).unsqueeze(0).clamp(0.0, 1.0)
    C = x.shape[1]
    w = window.expand(C, 1, *window.shape).contiguous()
    mu_x = F.conv2d(x, w, groups=C)
    mu_y = F.conv2d(y, w, groups=C)
    sxx = (F.conv2d(x * x, w, groups=C) - mu_x * mu_x).clamp(min=0.0)
    syy = (F.conv2d(y * y, w, groups=C) - mu_y * mu_y).clamp(min=0.0)
    sxy = F.conv2d(x * y, w, groups=C) - mu_x * mu_y
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    num = (2 * mu_x * mu_y + c1) * (2 * sxy + c2)
    den = (mu_x * mu_x + mu_y * mu_y + c1) * (sxx + syy + c2)
    return (num / den).mean()


def reconstruction_loss(img: torch.Tensor, target: torch.Tensor, window: torch.Tensor) -> torch.Tensor:
    l1 = (img - target).abs().mean()
    return (1.0 - LAMBDA_DSSIM) * l1 + LAMBDA_DSSIM * (1.0 - ssim(img, target, window))


@dataclass
class ShardPlan:
    """Which views of a batch of `batch` a rank renders."""

    rank: int
    world: int
    batch: int

    def views(self) -> list[int]:
        return list(range(self.rank, self.batch, self.world))


class FlatGrads:
    """One contiguous fp32 buffer backing the .grad of every parameter, followed (at
    `stats_offset`, default right after the gradients) by the densification sums (per Gaussian:
    norm sum, count). `buffer` / `max_grad` may be given (the sharded step's symmetric
    buffers); otherwise they are allocated here."""

    def __init__(self, params: list[torch.Tensor], n_gaussians: int, buffer=None,
                 stats_offset: int | None = None, max_grad=None):
        sizes = [p.numel() for p in params]
        self.n_param = sum(sizes)
        self.n = n_gaussians
        dev = params[0].device
        so = self.n_param if stats_offset is None else stats_offset
        if buffer is None:
            buffer = torch.zeros(so + 2 * n_gaussians, device=dev, dtype=torch.float32)
        if buffer.numel() < so + 2 * n_gaussians or so < self.n_param:
            raise ValueError("gradient bucket too small for the parameters and statistics")
        self.buffer = buffer
        off = 0
        self.views = []
        for p, k in zip(params, sizes):
            v = self.buffer[off:off + k].view_as(p)
            p.grad = v
            self.views.append(v)
            off += k
        self.grad_norm_sum = self.buffer[so:so + n_gaussians]
        self.grad_count = self.buffer[so + n_gaussians:so + 2 * n_gaussians]
        self.max_grad = (torch.zeros(n_gaussians, device=dev, dtype=torch.float32)
                         if max_grad is None else max_grad)

    def zero(self) -> None:
        self.buffer.zero_()
        self.max_grad.zero_()

    def zero_stats(self) -> None:
        """Clears the densification statistics only (sums, counts, maxima)."""
        self.grad_norm_sum.zero_()
        self.grad_count.zero_()
        self.max_grad.zero_()

    def rebind(self, params: list[torch.Tensor]) -> None:
        for p, v in zip(params, self.views):
            p.grad = v


def accumulate_view_stats(fg: FlatGrads, mean2d_grad: torch.Tensor, width: int,
                          height: int) -> None:
    """adc.py:58-80 statistics for one view: ||dL/dmean2d * (W/2, H/2)|| summed and counted
    where non-zero, and its running maximum."""
    scale = torch.tensor([width / 2.0, height / 2.0], device=mean2d_grad.device)
    norm = (mean2d_grad[:, :2] * scale).norm(dim=-1)
    visible = norm > 0
    fg.grad_norm_sum.add_(torch.where(visible, norm, torch.zeros_like(norm)))
    fg.grad_count.add_(visible.to(norm.dtype))
    torch.maximum(fg.max_grad, norm, out=fg.max_grad)


def reduce_step(fg: FlatGrads, batch: int, world: int, group=None) -> None:
    """Batch-mean gradients and the densification statistics across ranks."""
    if world > 1:
        dist.all_reduce(fg.buffer, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(fg.max_grad, op=dist.ReduceOp.MAX, group=group)
    fg.buffer[:fg.n_param].div_(float(batch))


class HostTargets:
    """Target images kept in pinned host memory and staged to the device every step.

    `issue()` enqueues this step's host->device copies on a side stream, one per view, into
    per-view device buffers; `get(vi)` makes the compute stream wait for view vi's copy only,
    so the copies overlap the rendering of earlier views; `release(vi)` marks the buffer as
    consumed by this step's loss, and the next step's copy into it waits for that mark.
    """

    def __init__(self, host: dict, device: torch.device):
        self.host = host
        self.dev = {vi: torch.empty(h.shape, dtype=h.dtype, device=device) for vi, h in host.items()}
        self.stream = torch.cuda.Stream(device)
        self.copied = {vi: torch.cuda.Event() for vi in host}
        self.consumed = {vi: None for vi in host}

    @property
    def bytes_per_step(self) -> int:
        return sum(h.numel() * h.element_size() for h in self.host.values())

    def issue(self) -> None:
        with torch.cuda.stream(self.stream):
            for vi, h in self.host.items():
                if self.consumed[vi] is not None:
                    self.stream.wait_event(self.consumed[vi])
                self.dev[vi].copy_(h, non_blocking=True)
                self.copied[vi].record(self.stream)

    def get(self, vi: int) -> torch.Tensor:
        torch.cuda.current_stream(self.stream.device).wait_event(self.copied[vi])
        return self.dev[vi]

    def release(self, vi: int) -> None:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.stream.device))
        self.consumed[vi] = ev


class Trainer:
    """Parameters, optimizer and flat gradient bucket of one rank.

    mode "direct" (default) calls the fused render and loss kernels without autograd: each
    view's parameter gradients are added straight into the flat bucket, the densification
    statistics are updated inside the per-Gaussian backward kernel and the opacity gradient is
    taken through the sigmoid once per step. Consecutive views run on `view_streams`
    alternating CUDA streams (1 = all on the current stream), the blend kernels then in their
    throughput variants (GS_RENDER_CONCURRENT) when the rank has more than one view of the
    batch; with several views the per-Gaussian half of the backward runs once per step over all
    of them (`combined_backward`), and with `tight_bins` the splats are binned
    only into tiles where they can pass the opacity test (same images and gradients, shorter
    tile lists). mode "autograd" runs the same step through
    `gaussian_splatting.rasterizer.rasterize` (the drop-in RasterizeFunction) and
    loss.backward(), as the reference trainer does.
    """

    def __init__(self, scene, views, targets, device, rank=0, world=1, group=None,
                 fused_adam: bool = True, fused_loss: bool = True, mode: str = "direct",
                 view_streams: int = 8, tight_bins: bool = True,
                 param_clamps: dict | None = None, combined_backward: bool = True):
        from gaussian_splatting.scene.gaussian import gaussian

        self.device = device
        self.rank, self.world, self.group = rank, world, group
        g = gaussian(scene.N)
        lrs = [LEARNING_RATES[n] for n in PARAM_NAMES]
        # several CUDA ranks: parameters, gradients and statistics in symmetric memory, and one
        # fused reduce-scatter + Adam + all-gather kernel per step (gs3d_b200.sharded)
        self.sharded = None
        if world > 1 and device.type == "cuda" and fused_adam:
            from gs3d_b200.sharded import ShardedStep

            self.sharded = ShardedStep(list(scene.params()), list(PARAM_NAMES), lrs, scene.N,
                                       len(views), device, group, eps=1e-15)
            for name, v in zip(PARAM_NAMES, self.sharded.param_views):
                setattr(g, name, torch.nn.Parameter(v))
        else:
            for name, t in zip(PARAM_NAMES, scene.params()):
                setattr(g, name, torch.nn.Parameter(t.to(device).contiguous()))
        self.gaussians = g
        self.params = [getattr(g, n) for n in PARAM_NAMES]
        self.views = [v.as_dict(device) for v in views]
        self.targets = targets
        self.plan = ShardPlan(rank, world, len(views))
        self.window = gaussian_window(device=device)
        if self.sharded is not None:
            self.fg = FlatGrads(self.params, scene.N, buffer=self.sharded.bucket,
                                stats_offset=self.sharded.layout.stats_offset,
                                max_grad=self.sharded.max_stat)
            self.opt = self.sharded
        elif fused_adam and device.type == "cuda":
            from gs3d_b200.optim import FlatAdam

            self.fg = FlatGrads(self.params, scene.N)
            self.opt = FlatAdam(self.params, lrs, list(PARAM_NAMES), self.fg.buffer, eps=1e-15)
        else:
            self.fg = FlatGrads(self.params, scene.N)
            groups = [{"params": [getattr(g, n)], "lr": LEARNING_RATES[n], "name": n}
                      for n in PARAM_NAMES]
            self.opt = torch.optim.Adam(groups, lr=0.0, eps=1e-15)
        # optional clamps after each update, by attribute name (gs3d_b200.clamps); the fused
        # optimizers apply them in their own pass
        self.param_clamps = dict(param_clamps or {})
        for grp in self.opt.param_groups:
            if grp["name"] in self.param_clamps:
                grp["clamp"] = self.param_clamps[grp["name"]]
        self.fused_loss = fused_loss and device.type == "cuda"
        if mode not in ("direct", "autograd"):
            raise ValueError(f"unknown trainer mode {mode!r}")
        self.mode = mode
        self.cam_positions = [(-torch.matmul(v["R"].T, v["T"])).reshape(3).contiguous()
                              for v in self.views]
        self.g_opacity = torch.zeros(scene.N, device=device, dtype=torch.float32)
        self.tight_bins = tight_bins
        self._streams, self._accum_events = [], []
        if mode == "direct" and device.type == "cuda" and view_streams > 1:
            from custom_rasterizer_cuda import _lib

            with torch.cuda.device(device):
                self._streams = [torch.cuda.Stream(device) for _ in range(view_streams)]
                self._accum_events = [_lib.Event(), _lib.Event()]
        # views overlap on streams: the blend kernels' throughput variants (also in steps
        # whose views run in order, so that per-stage timings see the same kernels). A rank
        # with one view of the batch overlaps nothing and takes the single-view variants: alone
        # their time varies less with the view (on B200, across config-4 views, backward
        # 0.79-0.80 ms against 0.73-0.96 ms for the four-pixel variant), and the step waits for
        # the slowest rank.
        self.concurrent_views = len(self._streams) > 1 and len(self.plan.views()) > 1
        # the per-Gaussian half of the backward once per step over all of the rank's views
        # (parameters read and gradients written once) instead of once per view; each view's
        # blend sums wait in their own buffer until then (same bits as per view, in view order;
        # on B200 the 8-view config-4 step 11.89 -> 11.30 ms, 2 views 3.41 -> 3.34 ms; with one
        # view the single-view kernel is slightly faster and stays)
        self.combined_backward = (combined_backward and mode == "direct"
                                  and len(self.plan.views()) > 1)
        self._sums = []

    def _update(self) -> None:
        """Batch-mean gradients across ranks, then Adam. The sharded step does both (and the
        statistic reductions) in its one kernel; otherwise reduce_step + the optimizer."""
        if self.sharded is None:
            reduce_step(self.fg, len(self.views), self.world, self.group)
        self.opt.step()
        if isinstance(self.opt, torch.optim.Optimizer):  # torch's Adam: clamps as torch ops
            with torch.no_grad():
                for grp in self.opt.param_groups:
                    lo, hi = grp.get("clamp") or (None, None)
                    if lo is not None or hi is not None:
                        grp["params"][0].clamp_(lo, hi)

    def step(self, targets=None, before_view=None) -> torch.Tensor:
        if self.mode == "direct":
            return self._step_direct(targets, before_view)
        return self._step_autograd(targets, before_view)

    def _step_direct(self, targets=None, before_view=None) -> torch.Tensor:
        """One step with the fused kernels called directly (see the class docstring)."""
        from custom_rasterizer_cuda.render import render_backward, render_forward
        from gs3d_b200.loss import l1_ssim_value_and_grad

        targets = self.targets if targets is None else targets
        staged = isinstance(targets, HostTargets)
        if staged:
            targets.issue()
        g = self.gaussians
        fg = self.fg
        fg.rebind(self.params)
        views = self.plan.views()
        if views:
            # the first view's backward overwrites every parameter gradient (and g_opacity), so
            # only the statistics and the opacity-logit slice (written through the sigmoid
            # below) need clearing
            fg.zero_stats()
            g.alpha.grad.zero_()
        else:
            fg.zero()
            self.g_opacity.zero_()
        with torch.no_grad():
            mu, q, s, A, kj = g.mu.detach(), g.q.detach(), g.s.detach(), g.A.detach(), g.k_j.detach()
            opacity = torch.sigmoid(g.alpha.detach()).reshape(-1)
            out = (g.mu.grad, g.q.grad, g.s.grad, self.g_opacity, g.A.grad, g.k_j.grad)
            main = torch.cuda.current_stream(self.device)
            # consecutive views on alternating streams (unless a per-view hook wants them in
            # order): a view's forward overlaps the previous view's loss and backward; only the
            # kernels that add into the shared gradient bucket are chained across streams
            streams = self._streams if (self._streams and before_view is None) else [main]
            for st in streams:
                if st is not main:
                    st.wait_stream(main)
            # The host does not wait for any view's pair count here: each view's pair buffers
            # are sized from the last pair count seen (+12.5%), and all views are checked once
            # below, before the update. A view whose pairs overflowed its buffers rendered
            # nothing (its blend kernels and backward do no work, adding zero gradients) and is
            # rendered again with exact buffers.
            combined = self.combined_backward
            if combined:
                from custom_rasterizer_cuda.render import (backward_workspace,
                                                           backward_workspace_bytes,
                                                           render_backward_blend,
                                                           render_backward_views)
                n_g = g.mu.shape[0]
                self._sums = [ws if ws.numel() >= backward_workspace_bytes(n_g) else
                              backward_workspace(n_g, self.device) for ws in self._sums]
                while len(self._sums) < len(views):
                    self._sums.append(backward_workspace(n_g, self.device))

            def render_view(k, vi, st, done, prev_done, capacity=None, accumulate=None):
                v = self.views[vi]
                cam = self.cam_positions[vi]
                with torch.cuda.stream(st):
                    img, _, rs = render_forward(mu, q, s, opacity, A, kj, v["R"], v["T"], cam,
                                                v["fx"], v["fy"], v["cx"], v["cy"], v["height"],
                                                v["width"], tight_bins=self.tight_bins,
                                                concurrent=self.concurrent_views,
                                                defer_check=True, capacity=capacity)
                    target = targets.get(vi) if staged else targets[vi]
                    loss, gimg = l1_ssim_value_and_grad(img, target, LAMBDA_DSSIM)
                    if staged:  # the next step's copy into this target waits for this point
                        targets.release(vi)
                    if combined:
                        render_backward_blend(rs, gimg, mu.shape[0], self._sums[k])
                        return loss, rs
                    render_backward(rs, gimg, mu, q, s, A, kj, v["R"], v["T"], cam, v["fx"],
                                    v["fy"], v["cx"], v["cy"], want_mean2d_grad=False, out=out,
                                    stats=(fg.grad_norm_sum, fg.grad_count, fg.max_grad,
                                           v["width"] / 2.0, v["height"] / 2.0),
                                    accum_wait=prev_done, accum_done=done,
                                    accumulate=(k > 0) if accumulate is None else accumulate)
                return loss, rs

            losses, states, prev_done = [], [], None
            for k, vi in enumerate(views):
                if before_view is not None:
                    before_view(vi)
                st = streams[k % len(streams)]
                done = self._accum_events[k % 2] if len(streams) > 1 else None
                loss, rs = render_view(k, vi, st, done, prev_done)
                prev_done = done
                if st is not main:
                    loss.record_stream(main)
                losses.append(loss)
                states.append(rs)
            for st in streams:
                if st is not main:
                    main.wait_stream(st)
            for k, (vi, rs) in enumerate(zip(views, states)):
                if rs.overflowed():
                    loss, rs2 = render_view(k, vi, main, None, None, capacity=rs.pairs,
                                            accumulate=True)
                    if rs2.overflowed():
                        raise RuntimeError("pair count changed between two renders of a view")
                    losses[k] = loss
            if combined and views:
                render_backward_views(
                    [(self._sums[k], self.views[vi]["R"], self.views[vi]["T"],
                      self.cam_positions[vi], self.views[vi]["fx"], self.views[vi]["fy"],
                      self.views[vi]["cx"], self.views[vi]["cy"], self.views[vi]["width"] / 2.0,
                      self.views[vi]["height"] / 2.0) for k, vi in enumerate(views)],
                    mu, q, s, A, kj, out,
                    stats=(fg.grad_norm_sum, fg.grad_count, fg.max_grad))
            total = torch.stack(losses).sum() if losses else torch.zeros((), device=self.device)
            # d loss / d logit = d loss / d opacity * sigmoid'(logit), once per step
            g.alpha.grad.view(-1).addcmul_(self.g_opacity, opacity * (1.0 - opacity))
        self._update()
        return total

    def _step_autograd(self, targets=None, before_view=None) -> torch.Tensor:
        """One training step over this rank's share of the batch; returns the summed loss of
        the local views (a 0-d tensor on the device). `before_view(vi)`, if given, is called
        before view vi is rendered (the benchmark installs its stage events there)."""
        from gaussian_splatting.rasterizer.rasterize import RasterizeFunction, rasterize

        targets = self.targets if targets is None else targets
        staged = isinstance(targets, HostTargets)
        if staged:
            targets.issue()
        self.fg.zero()
        self.fg.rebind(self.params)
        total = torch.zeros((), device=self.device)
        for vi in self.plan.views():
            view = self.views[vi]
            if before_view is not None:
                before_view(vi)
            img = rasterize(self.gaussians, view)
            target = targets.get(vi) if staged else targets[vi]
            if self.fused_loss:
                from gs3d_b200.loss import l1_ssim_loss

                loss = l1_ssim_loss(img, target, LAMBDA_DSSIM)
            else:
                loss = reconstruction_loss(img, target, self.window)
            loss.backward()
            if staged:
                targets.release(vi)
            accumulate_view_stats(self.fg, RasterizeFunction.last_mean2d_grad, view["width"],
                                  view["height"])
            total = total + loss.detach()
        self._update()
        return total
