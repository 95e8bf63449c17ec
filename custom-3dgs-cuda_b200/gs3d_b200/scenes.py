"""Seeded synthetic scenes of the benchmark configurations (configs 0-4) and of the
reference's own scripts/bench.py scene.

Every scene is drawn on the CPU with torch.Generator("cpu").manual_seed(seed) in the order
means, log-scales, quaternions, opacity logits, SH (DC then degrees 1-3), so a seed gives the
same scene on every machine. Cameras use the OpenCV convention the reference expects
(x right, y down, z forward; world-to-camera R, t).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class View:
    R: torch.Tensor          # [3,3] world -> camera
    T: torch.Tensor          # [3]
    fx: float
    fy: float
    cx: float
    cy: float
    height: int
    width: int

    def as_dict(self, device=None) -> dict:
        d = dict(R=self.R, T=self.T, fx=self.fx, fy=self.fy, cx=self.cx, cy=self.cy,
                 height=self.height, width=self.width)
        if device is not None:
            d["R"] = self.R.to(device)
            d["T"] = self.T.to(device)
        return d


@dataclass
class Scene:
    name: str
    mu: torch.Tensor
    q: torch.Tensor
    s: torch.Tensor
    alpha: torch.Tensor      # opacity logits [N,1]
    A: torch.Tensor          # SH DC [N,3]
    k_j: torch.Tensor        # SH degrees 1..3 [N,15,3]
    views: list[View] = field(default_factory=list)

    @property
    def N(self) -> int:
        return int(self.mu.shape[0])

    def params(self) -> tuple[torch.Tensor, ...]:
        return (self.mu, self.q, self.s, self.alpha, self.A, self.k_j)

    def to(self, device) -> "Scene":
        return Scene(self.name, *(p.to(device) for p in self.params()), views=self.views)


def look_at(eye, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)) -> tuple[torch.Tensor, torch.Tensor]:
    """World-to-camera (R, t) of a camera at `eye` looking at `target` (x right, y down)."""
    eye = torch.tensor(eye, dtype=torch.float64)
    f = torch.tensor(target, dtype=torch.float64) - eye
    f = f / f.norm()
    upv = torch.tensor(up, dtype=torch.float64)
    if abs(float(f @ upv)) > 0.999:
        upv = torch.tensor((0.0, 0.0, 1.0), dtype=torch.float64)
    r = torch.linalg.cross(f, upv)
    r = r / r.norm()
    d = torch.linalg.cross(f, r)
    R = torch.stack([r, d, f])
    t = -(R @ eye)
    return R.float(), t.float()


def pinhole(eye, width, height, focal, target=(0.0, 0.0, 0.0)) -> View:
    R, t = look_at(eye, target)
    return View(R, t, float(focal), float(focal), width * 0.5, height * 0.5, int(height), int(width))


def _draw(gen, n, means, logscale_mu, logscale_sigma, opacity_sigma=1.0):
    s = torch.randn(n, 3, generator=gen) * logscale_sigma + logscale_mu
    q = torch.randn(n, 4, generator=gen)
    q = q / q.norm(dim=1, keepdim=True)
    alpha = torch.randn(n, 1, generator=gen) * opacity_sigma
    A = torch.randn(n, 3, generator=gen) * 0.5
    k_j = torch.randn(n, 15, 3, generator=gen) * 0.05
    return means.float(), q.float(), s.float(), alpha.float(), A.float(), k_j.float()


def config0(seed: int = 0) -> Scene:
    """4,096 Gaussians in [-1,1]^3, log-scales N(-4, 0.5), 128x128, f=128, camera at z=4."""
    g = torch.Generator("cpu").manual_seed(seed)
    n = 4096
    means = torch.rand(n, 3, generator=g) * 2.0 - 1.0
    sc = Scene("config0", *_draw(g, n, means, -4.0, 0.5))
    sc.views = [pinhole((0.0, 0.0, 4.0), 128, 128, 128.0)]
    return sc


def config1(seed: int = 0) -> Scene:
    """100k Gaussians in [-2,2]^3; views 1280x720 (f=1000) and 1920x1080 (f=1500) at z=6."""
    g = torch.Generator("cpu").manual_seed(seed)
    n = 100_000
    means = torch.rand(n, 3, generator=g) * 4.0 - 2.0
    sc = Scene("config1", *_draw(g, n, means, -4.0, 0.5))
    sc.views = [pinhole((0.0, 0.0, 6.0), 1280, 720, 1000.0),
                pinhole((0.0, 0.0, 6.0), 1920, 1080, 1500.0)]
    return sc


def clustered_means(g: torch.Generator, n: int, components: int = 64) -> torch.Tensor:
    """Isotropic Gaussian mixture: centres U[-3,3]^3, per-component sigma U[0.05, 0.5]."""
    centers = torch.rand(components, 3, generator=g) * 6.0 - 3.0
    sigmas = torch.rand(components, generator=g) * 0.45 + 0.05
    comp = torch.randint(0, components, (n,), generator=g)
    return centers[comp] + torch.randn(n, 3, generator=g) * sigmas[comp, None]


def config2(seed: int = 0, n: int = 1_000_000) -> Scene:
    """1M clustered Gaussians, log-scales N(-4.5, 0.7), opacity logits N(0, 1.5), 1080p at z=8."""
    g = torch.Generator("cpu").manual_seed(seed)
    means = clustered_means(g, n)
    sc = Scene("config2", *_draw(g, n, means, -4.5, 0.7, opacity_sigma=1.5))
    sc.views = [pinhole((0.0, 0.0, 8.0), 1920, 1080, 1500.0)]
    return sc


def config3(seed: int = 0, n: int = 3_000_000, n_views: int = 32) -> Scene:
    """3M Gaussians in [-4,4]^3, log-scales N(-5, 0.7); 4K views on a great circle, r=10."""
    g = torch.Generator("cpu").manual_seed(seed)
    means = torch.rand(n, 3, generator=g) * 8.0 - 4.0
    sc = Scene("config3", *_draw(g, n, means, -5.0, 0.7))
    sc.views = []
    for k in range(n_views):
        a = 2.0 * math.pi * k / n_views
        sc.views.append(pinhole((10.0 * math.sin(a), 0.0, 10.0 * math.cos(a)), 3840, 2160, 3000.0))
    return sc


def config4(seed: int = 0, n: int = 1_000_000, n_views: int = 8) -> tuple[Scene, list[torch.Tensor]]:
    """Config-2 Gaussians with 8 seeded 1080p views on a sphere of radius 8, and seeded
    uniform[0,1] target images."""
    sc = config2(seed, n)
    sc.name = "config4"
    g = torch.Generator("cpu").manual_seed(seed + 1)
    sc.views = []
    targets = []
    for _ in range(n_views):
        d = torch.randn(3, generator=g, dtype=torch.float64)
        d = d / d.norm() * 8.0
        sc.views.append(pinhole(tuple(float(v) for v in d), 1920, 1080, 1500.0))
        targets.append(torch.rand(1080, 1920, 3, generator=g))
    return sc, targets


def reference_bench_scene(n: int = 100_000, seed: int = 0, width: int = 1280,
                          height: int = 720) -> Scene:
    """The reference's scripts/bench.py scene (bench.py:30-63): z ~ U[2,6], x, y scaled by z,
    identity rotation, log-scale -3, opacity logit 0, zero SH; identity camera, f = width."""
    g = torch.Generator("cpu").manual_seed(seed)
    z = torch.empty(n, 1).uniform_(2.0, 6.0, generator=g)
    x = torch.empty(n, 1).uniform_(-0.35, 0.35, generator=g) * z
    y = torch.empty(n, 1).uniform_(-0.25, 0.25, generator=g) * z
    q = torch.zeros(n, 4)
    q[:, 0] = 1.0
    sc = Scene("reference_bench", torch.cat((x, y, z), 1), q, torch.full((n, 3), -3.0),
               torch.zeros(n, 1), torch.zeros(n, 3), torch.zeros(n, 15, 3))
    sc.views = [View(torch.eye(3), torch.zeros(3), float(width), float(width), width * 0.5,
                     height * 0.5, height, width)]
    return sc


CONFIGS = {"config0": config0, "config1": config1, "config2": config2, "config3": config3}
