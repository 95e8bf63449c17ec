"""Per-group parameter clamps of the fused optimizer steps (gs_adam_step, gs_sharded_adam_step):
the reference trainer clamps the opacity logits to [logit(1e-4), logit(0.99)] and the
log-scales to at most log(0.1 * scene extent) right after optimizer.step()
(scripts/train.py:171-178); a param group's optional "clamp": (lo, hi) entry asks the step to
do the same in its pass."""

from __future__ import annotations

import ctypes
import math


def clamp_arrays(param_groups) -> tuple:
    """Host (clamp_min, clamp_max) float arrays from the groups' optional "clamp" entries, or
    (None, None) when no group is clamped."""
    bounds = [g.get("clamp") for g in param_groups]
    if all(b is None for b in bounds):
        return None, None
    inf = float("inf")
    lo = [(-inf if b is None or b[0] is None else float(b[0])) for b in bounds]
    hi = [(inf if b is None or b[1] is None else float(b[1])) for b in bounds]
    return (ctypes.c_float * len(lo))(*lo), (ctypes.c_float * len(hi))(*hi)


def reference_trainer_clamps(scene_extent: float) -> dict[str, tuple[float | None, float | None]]:
    """The reference trainer's clamps, keyed by Gaussian attribute ("alpha" is the reference's
    "Opacity" group, "s" its "Scale" group)."""
    return {"alpha": (math.log(1e-4 / (1.0 - 1e-4)), math.log(0.99 / (1.0 - 0.99))),
            "s": (None, math.log(max(0.1 * scene_extent, 1e-7)))}
