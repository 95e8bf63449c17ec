"""The PLY export packs on the parameters' device: a model on the GPU gives the same file as the
same model on the CPU."""

from __future__ import annotations

import pytest
import torch

from test_ply_io import make_gaussians

pytestmark = pytest.mark.gpu


def test_gpu_pack_matches_cpu(cuda_device, tmp_path):
    from gaussian_splatting.utils.ply import load_ply, pack_inria, save_ply

    cpu = make_gaussians(n=20_000, seed=4)
    gpu = make_gaussians(n=20_000, seed=4)
    for name in ("mu", "q", "s", "alpha", "A", "k_j"):
        setattr(gpu, name, getattr(gpu, name).to(cuda_device))
    a, b = pack_inria(cpu), pack_inria(gpu)
    assert b.device.type == "cuda"
    torch.testing.assert_close(b.cpu(), a, rtol=1e-6, atol=1e-7)
    save_ply(gpu, tmp_path / "g.ply")
    back = load_ply(tmp_path / "g.ply", device=cuda_device)
    assert torch.equal(back.k_j.cpu(), cpu.k_j) and torch.equal(back.mu.cpu(), cpu.mu)
