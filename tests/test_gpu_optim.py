"""FlatAdam (one gs_adam_step launch over all parameter groups) against torch.optim.Adam with
the reference trainer's settings (eps 1e-15, per-group learning rates): parameters and both
moments agree after several steps, for float4-aligned groups and for groups whose slices of
the flat buffers are misaligned (scalar path)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sizes", [(12, 4000, 36), (7, 1001, 3, 50_001)])
def test_flat_adam_matches_torch_adam(cuda_device, sizes):
    from gs3d_b200.optim import FlatAdam

    g = torch.Generator("cpu").manual_seed(sum(sizes))
    lrs = [1.6e-4, 5e-2, 2.5e-3, 1e-3][:len(sizes)]
    init = [torch.randn(k, generator=g) for k in sizes]
    mine = [t.clone().to(cuda_device) for t in init]
    ref = [t.clone().to(cuda_device).requires_grad_(True) for t in init]
    flat = torch.zeros(sum(sizes) + 5, device=cuda_device)
    off = 0
    for p, k in zip(mine, sizes):
        p.grad = flat[off:off + k]
        off += k
    opt = FlatAdam(mine, lrs, [f"g{i}" for i in range(len(sizes))], flat, eps=1e-15)
    torch_opt = torch.optim.Adam([{"params": [p], "lr": lr} for p, lr in zip(ref, lrs)],
                                 lr=0.0, eps=1e-15)
    for step in range(6):
        grads = [torch.randn(k, generator=g).to(cuda_device) * (10.0 ** (step % 3 - 1))
                 for k in sizes]
        off = 0
        for k, gr in zip(sizes, grads):
            flat[off:off + k] = gr
            off += k
        for p, gr in zip(ref, grads):
            p.grad = gr.clone()
        opt.step()
        torch_opt.step()
    torch.cuda.synchronize()
    for p, r in zip(mine, ref):
        torch.testing.assert_close(p, r.detach(), rtol=1e-6, atol=1e-6)
        st, rs = opt.state[p], torch_opt.state[r]
        # moments of O(1..10) values: a few float32 ulps of rounding-order difference
        torch.testing.assert_close(st["exp_avg"], rs["exp_avg"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(st["exp_avg_sq"], rs["exp_avg_sq"], rtol=1e-5, atol=1e-6)
        assert st["step"] == 6


def test_flat_adam_clamps_like_torch_clamp_after_step(cuda_device):
    """A group's "clamp" bounds give the same parameters as torch Adam followed by clamp_ (the
    reference trainer's opacity / log-scale clamps), unclamped groups are untouched."""
    from gs3d_b200.optim import FlatAdam

    g = torch.Generator("cpu").manual_seed(3)
    sizes, lrs = (5000, 3000, 700), [5e-2, 5e-3, 1e-3]
    clamps = [(-0.5, 0.5), (None, 0.25), None]
    init = [torch.randn(k, generator=g) for k in sizes]
    mine = [t.clone().to(cuda_device) for t in init]
    ref = [t.clone().to(cuda_device).requires_grad_(True) for t in init]
    flat = torch.zeros(sum(sizes), device=cuda_device)
    off = 0
    for p, k in zip(mine, sizes):
        p.grad = flat[off:off + k]
        off += k
    opt = FlatAdam(mine, lrs, ["alpha", "s", "q"], flat, eps=1e-15)
    for grp, c in zip(opt.param_groups, clamps):
        if c is not None:
            grp["clamp"] = c
    torch_opt = torch.optim.Adam([{"params": [p], "lr": lr} for p, lr in zip(ref, lrs)],
                                 lr=0.0, eps=1e-15)
    for _ in range(4):
        grads = [torch.randn(k, generator=g).to(cuda_device) for k in sizes]
        flat.copy_(torch.cat(grads))
        for p, gr in zip(ref, grads):
            p.grad = gr.clone()
        opt.step()
        torch_opt.step()
        with torch.no_grad():
            for p, c in zip(ref, clamps):
                if c is not None:
                    p.clamp_(*c)
    torch.cuda.synchronize()
    for p, r, c in zip(mine, ref, clamps):
        torch.testing.assert_close(p, r.detach(), rtol=1e-6, atol=1e-6)
        if c is not None:
            lo = -float("inf") if c[0] is None else c[0]
            assert float(p.min()) >= lo and float(p.max()) <= c[1]
            assert bool((p == c[1]).any())  # the bound was reached


def test_flat_adam_rejects_grads_outside_the_buffer(cuda_device):
    from gs3d_b200.optim import FlatAdam

    p = torch.zeros(8, device=cuda_device)
    p.grad = torch.zeros(8, device=cuda_device)
    with pytest.raises(ValueError):
        FlatAdam([p], [1e-3], ["p"], torch.zeros(8, device=cuda_device))
