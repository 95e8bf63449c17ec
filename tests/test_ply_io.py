"""On-disk formats (CPU): the Inria `point_cloud.ply` export of the reference's `save_ply`
(scripts/run.py:66-165) and the `.pt` checkpoints of its `save_weights` / `load_gaussians`
(gaussian_splatting/utils/saveweights.py, scripts/run.py:56-63). The PLY layout is checked
against the reference's property list and transforms restated here with numpy; `plyfile`, which
the reference writes through, is not installed, so the byte-level header is the PLY standard's
(binary_little_endian, `property float <name>` per attribute)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

NAMES = ("mu", "q", "s", "alpha", "A", "k_j")


def make_gaussians(n=257, seed=0, opacity_probs=False):
    from gaussian_splatting.scene.gaussian import gaussian

    g = torch.Generator().manual_seed(seed)
    gs = gaussian(n)
    gs.mu = torch.randn(n, 3, generator=g)
    gs.q = torch.randn(n, 4, generator=g) * 2.0
    gs.s = torch.randn(n, 3, generator=g) - 4.0
    gs.alpha = (torch.rand(n, 1, generator=g) * 0.9 + 0.05 if opacity_probs
                else torch.randn(n, 1, generator=g) * 2.0)
    gs.A = torch.randn(n, 3, generator=g)
    gs.k_j = torch.randn(n, 15, 3, generator=g) * 0.1
    return gs


def expected_rows(gs):
    """The reference exporter's transforms, restated with numpy."""
    n = gs.mu.shape[0]
    q = gs.q.numpy()
    qn = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), 1e-8)
    a = gs.alpha.numpy().reshape(n, 1)
    if ((a > 0) & (a < 1)).all() and a.min() > 1e-6:
        a = np.clip(a, 1e-6, 1 - 1e-6)
        a = np.log(a / (1 - a))
    rest = gs.k_j.numpy().transpose(0, 2, 1).reshape(n, 45)
    return np.concatenate([gs.mu.numpy(), np.zeros((n, 3), np.float32), gs.A.numpy(), rest, a,
                           gs.s.numpy(), qn], axis=1).astype(np.float32)


def test_ply_layout_and_values(tmp_path):
    from gaussian_splatting.utils.ply import ply_property_names, read_ply_vertices, save_ply

    gs = make_gaussians()
    path = tmp_path / "out" / "point_cloud.ply"
    save_ply(gs, path)
    names = ply_property_names()
    assert names[:9] == ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"]
    assert names[9:54] == [f"f_rest_{i}" for i in range(45)]
    assert names[54:] == ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1",
                          "rot_2", "rot_3"]
    data = path.read_bytes()
    header = data[:data.index(b"end_header\n") + len(b"end_header\n")].decode()
    assert header.splitlines()[:3] == ["ply", "format binary_little_endian 1.0",
                                       f"element vertex {gs.mu.shape[0]}"]
    assert header.splitlines()[3:-1] == [f"property float {n}" for n in names]
    assert len(data) == len(header) + gs.mu.shape[0] * 62 * 4
    v = read_ply_vertices(path)
    got = np.stack([v[n] for n in names], axis=1)
    np.testing.assert_allclose(got, expected_rows(gs), rtol=1e-6, atol=1e-7)
    # f_rest is channel-major: f_rest_{15 c + k} = k_j[:, k, c]
    np.testing.assert_array_equal(v["f_rest_16"], gs.k_j[:, 1, 1].numpy())


def test_ply_round_trip_and_legacy_opacity(tmp_path):
    from gaussian_splatting.utils.ply import load_ply, save_ply

    gs = make_gaussians(seed=1)
    save_ply(gs, tmp_path / "a.ply")
    back = load_ply(tmp_path / "a.ply")
    for name in ("mu", "s", "alpha", "A", "k_j"):
        assert torch.equal(getattr(back, name), getattr(gs, name).reshape(getattr(back, name).shape))
    qn = gs.q / gs.q.norm(dim=-1, keepdim=True).clamp_min(1e-8)
    torch.testing.assert_close(back.q, qn, rtol=1e-6, atol=1e-7)
    # a legacy checkpoint that stores probabilities is written as logits
    legacy = make_gaussians(seed=2, opacity_probs=True)
    save_ply(legacy, tmp_path / "b.ply")
    p = legacy.alpha.numpy()
    np.testing.assert_allclose(load_ply(tmp_path / "b.ply").alpha.numpy(),
                               np.log(p / (1 - p)), rtol=1e-5, atol=1e-6)


def test_ply_reader_rejects_other_formats(tmp_path):
    from gaussian_splatting.utils.ply import read_ply_vertices

    (tmp_path / "t.ply").write_bytes(b"ply\nformat ascii 1.0\nelement vertex 1\n"
                                     b"property float x\nend_header\n1.0\n")
    with pytest.raises(ValueError, match="unsupported"):
        read_ply_vertices(tmp_path / "t.ply")
    (tmp_path / "u.bin").write_bytes(b"nope")
    with pytest.raises(ValueError, match="not a PLY"):
        read_ply_vertices(tmp_path / "u.bin")


def test_checkpoint_round_trip_and_reference_dict(tmp_path):
    from gaussian_splatting.utils.saveweights import load_weights, save_weights

    gs = make_gaussians(seed=3)
    save_weights(gs, tmp_path / "ck" / "gaussians_final.pt")
    back = load_weights(tmp_path / "ck" / "gaussians_final.pt")
    assert back.N == gs.N
    for name in NAMES:
        assert torch.equal(getattr(back, name), getattr(gs, name))
    # a dict in the reference's checkpoint layout (parameters + "N") loads the same way
    ref = {name: getattr(gs, name).double() for name in NAMES}
    ref["N"] = gs.N
    torch.save(ref, tmp_path / "ref.pt")
    back = load_weights(tmp_path / "ref.pt")
    for name in NAMES:
        assert getattr(back, name).dtype == torch.float32
        torch.testing.assert_close(getattr(back, name), getattr(gs, name))
