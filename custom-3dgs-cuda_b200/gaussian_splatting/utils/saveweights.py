"""Gaussian checkpoints in the reference's `.pt` format (gaussian_splatting/utils/saveweights.py
and `load_gaussians` in scripts/run.py:56-63 of the reference): a torch.save'd dict of the six
parameter tensors on the CPU plus the Gaussian count "N"."""

from __future__ import annotations

from pathlib import Path

import torch

from gaussian_splatting.scene.gaussian import gaussian

_KEYS = ("mu", "q", "s", "alpha", "A", "k_j")


def save_weights(gaussians: gaussian, path) -> None:
    """Saves Gaussian parameters to a .pt checkpoint (parent directories created)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    state = {k: getattr(gaussians, k).detach().cpu() for k in _KEYS}
    state["N"] = gaussians.N
    torch.save(state, path)


def load_weights(path, device="cpu") -> gaussian:
    """Reads a checkpoint written by `save_weights` (or the reference's) into a `gaussian` with
    contiguous float32 tensors on `device`."""
    state = torch.load(path, map_location="cpu", weights_only=True)
    n = int(state["N"])
    g = gaussian(n)
    for k in _KEYS:
        setattr(g, k, state[k].to(device=device, dtype=torch.float32).contiguous())
    g.N = n
    return g
