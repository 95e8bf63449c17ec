"""Gaussian parameter container with the reference's field names and layouts
(gaussian_splatting/scene/gaussian.py:3-12)."""

import torch


class gaussian:  # noqa: N801 - reference class name
    def __init__(self, N: int) -> None:
        self.N = N
        self.mu = torch.zeros(N, 3, dtype=torch.float32)      # means
        self.q = torch.zeros(N, 4, dtype=torch.float32)       # quaternions (w, x, y, z)
        self.s = torch.zeros(N, 3, dtype=torch.float32)       # log-scales
        self.alpha = torch.zeros(N, 1, dtype=torch.float32)   # opacity logits
        self.A = torch.zeros(N, 3, dtype=torch.float32)       # SH DC ("albedo")
        self.k_j = torch.zeros(N, 15, 3, dtype=torch.float32) # SH degrees 1..3
