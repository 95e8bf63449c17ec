"""Adam over parameters whose gradients are consecutive slices of one flat buffer.

`FlatAdam` is torch.optim.Adam (amsgrad off, no weight decay; the reference's trainer builds
`torch.optim.Adam(params, lr=lr, eps=1e-15)`, gaussian_splatting/utils/optim.py:31) restricted to
that layout, so one `gs_adam_step` launch updates every group: parameters, gradients and both
moments are read and written once. It keeps torch's optimizer surface where the reference's
trainer touches it: `param_groups` (one per parameter, with "lr" and "name", so learning-rate
schedules work unchanged), `state[p]` with "step", "exp_avg" and "exp_avg_sq" (views into the
flat moment buffers), `step()` and `zero_grad()`. A group may also hold "clamp": (lo, hi) (None
or +-inf for an open side); the step then clamps that parameter in the same pass, as the
reference trainer clamps opacity logits and log-scales after `optimizer.step()`
(scripts/train.py:171-178).
"""

from __future__ import annotations

import ctypes

import torch

from custom_rasterizer_cuda import _lib

from .clamps import clamp_arrays


class FlatAdam:
    def __init__(self, params: list[torch.Tensor], lrs: list[float], names: list[str],
                 flat_grad: torch.Tensor, betas=(0.9, 0.999), eps: float = 1e-15):
        if len(params) > 8:
            raise ValueError("FlatAdam takes at most 8 parameter tensors")
        sizes = [p.numel() for p in params]
        n = sum(sizes)
        if flat_grad.numel() < n or flat_grad.dtype != torch.float32 or not flat_grad.is_cuda:
            raise ValueError("flat_grad must be a CUDA float32 buffer holding every gradient")
        off = 0
        for p, k in zip(params, sizes):
            if not (p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()):
                raise ValueError("parameters must be contiguous CUDA float32 tensors")
            if p.grad is None or p.grad.data_ptr() != flat_grad[off:off + k].data_ptr():
                raise ValueError("each parameter's .grad must be its slice of flat_grad")
            off += k
        self.params = list(params)
        self.flat_grad = flat_grad
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        dev = flat_grad.device
        self.exp_avg = torch.zeros(n, device=dev, dtype=torch.float32)
        self.exp_avg_sq = torch.zeros(n, device=dev, dtype=torch.float32)
        self.param_groups = [{"params": [p], "lr": float(lr), "name": name}
                             for p, lr, name in zip(params, lrs, names)]
        self.state = {}
        off = 0
        for p, k in zip(params, sizes):
            self.state[p] = {"step": 0, "exp_avg": self.exp_avg[off:off + k].view_as(p),
                             "exp_avg_sq": self.exp_avg_sq[off:off + k].view_as(p)}
            off += k
        self.n_steps = 0
        self._sizes = (ctypes.c_longlong * len(sizes))(*sizes)


    def step(self) -> None:
        self.n_steps += 1
        k = len(self.params)
        ptrs = (ctypes.c_void_p * k)(*[p.data_ptr() for p in self.params])
        lrs = (ctypes.c_float * k)(*[g["lr"] for g in self.param_groups])
        dev = self.flat_grad.device
        with torch.cuda.device(dev):
            _lib.check(_lib.lib.gs_adam_step(
                k, ptrs, self._sizes, lrs, self.flat_grad.data_ptr(), self.exp_avg.data_ptr(),
                self.exp_avg_sq.data_ptr(), self.betas[0], self.betas[1], self.eps, self.n_steps,
                *clamp_arrays(self.param_groups), torch.cuda.current_stream(dev).cuda_stream))
        for p in self.params:
            self.state[p]["step"] = self.n_steps

    def zero_grad(self, set_to_none: bool = False) -> None:
        self.flat_grad.zero_()
