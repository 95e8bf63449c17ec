"""Gaussian export / import in the Inria 3DGS `point_cloud.ply` layout, as the reference's
`save_ply` (scripts/run.py:66-165) writes it, without the `plyfile` dependency.

The file is a binary little-endian PLY with one `vertex` element of 62 float properties in
Inria's order: x y z, nx ny nz (zeros), f_dc_0..2, f_rest_0..44, opacity, scale_0..2, rot_0..3.
Values are the pre-activation parameters viewers expect, transformed as the reference does:
the SH rest coefficients k_j [N, 15, 3] are written channel-major (all 15 red, then green, then
blue: k_j.transpose(1, 2) flattened), the opacity stays a logit (unless every value lies in
(0, 1) with a minimum above 1e-6: then the values are probabilities from a legacy checkpoint
and are written as logits), log-scales stay log-scales and quaternions (w, x, y, z) are
L2-normalised with a 1e-8 floor on the norm.

The per-Gaussian packing (normalisation, transpose, concatenation) runs on the tensors' own
device, so a trained model on the GPU is packed there and crosses to the host in one copy of
N x 248 bytes.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

from gaussian_splatting.scene.gaussian import gaussian


def ply_property_names(max_sh_degree: int = 3) -> list[str]:
    """The vertex properties, in file order."""
    n_rest = (max_sh_degree + 1) ** 2 - 1
    names = ["x", "y", "z", "nx", "ny", "nz"]
    names += [f"f_dc_{i}" for i in range(3)]
    names += [f"f_rest_{i}" for i in range(3 * n_rest)]
    names.append("opacity")
    names += [f"scale_{i}" for i in range(3)]
    names += [f"rot_{i}" for i in range(4)]
    return names


def pack_inria(gaussians: gaussian, max_sh_degree: int = 3) -> torch.Tensor:
    """[N, 62] float32 rows in the file's property order, built on the parameters' device.

    The rows are allocated once and each property group is written into its own column block;
    the SH rest block is viewed as [N, 3, K] so the channel-major order comes from the
    destination's layout (missing bands stay zero, extra bands are dropped)."""
    n_rest = (max_sh_degree + 1) ** 2 - 1
    with torch.no_grad():
        mu = gaussians.mu.detach().float()
        n = int(mu.numel() // 3)
        sh = gaussians.k_j.detach().float()
        if sh.dim() != 3 or sh.shape[2] != 3:
            raise ValueError(f"k_j must be [N, K, 3] spherical-harmonic coefficients, got shape "
                             f"{tuple(sh.shape)}")
        rows = torch.zeros((n, 6 + 3 + 3 * n_rest + 1 + 3 + 4), device=mu.device)
        c = 0

        def block(width: int) -> torch.Tensor:
            nonlocal c
            view = rows[:, c:c + width]
            c += width
            return view

        block(3).copy_(mu.reshape(n, 3))
        block(3)  # normals: zero
        block(3).copy_(gaussians.A.detach().float().reshape(n, 3))
        k = min(int(sh.shape[1]), n_rest)
        block(3 * n_rest).view(n, 3, n_rest)[:, :, :k] = sh[:, :k, :].transpose(1, 2)
        alpha = gaussians.alpha.detach().float().reshape(n)
        legacy = False
        if n > 0:
            lo, hi = torch.aminmax(alpha)
            legacy = float(lo) > 1e-6 and float(hi) < 1.0  # probabilities, not logits
        block(1)[:, 0] = torch.logit(alpha, eps=1e-6) if legacy else alpha
        block(3).copy_(gaussians.s.detach().float().reshape(n, 3))
        block(4).copy_(F.normalize(gaussians.q.detach().float().reshape(n, 4), dim=1, eps=1e-8))
        return rows


def _header(n: int, names: list[str]) -> bytes:
    lines = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    lines += [f"property float {name}" for name in names]
    lines.append("end_header")
    return ("\n".join(lines) + "\n").encode("ascii")


def save_ply(gaussians: gaussian, out_path, *, max_sh_degree: int = 3) -> None:
    """Writes `out_path` (parent directories created) in the Inria layout."""
    out_path = Path(out_path)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    rows = pack_inria(gaussians, max_sh_degree)
    host = rows.cpu().numpy().astype("<f4", copy=False)
    names = ply_property_names(max_sh_degree)
    assert host.shape[1] == len(names)
    with open(out_path, "wb") as f:
        f.write(_header(host.shape[0], names))
        f.write(np.ascontiguousarray(host).tobytes())


def export_attributes(gaussians: gaussian, out_path) -> None:
    """Alias of `save_ply`, as in the reference."""
    save_ply(gaussians, out_path)


_PLY_TYPES = {"char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1", "short": "i2",
              "int16": "i2", "ushort": "u2", "uint16": "u2", "int": "i4", "int32": "i4",
              "uint": "u4", "uint32": "u4", "float": "f4", "float32": "f4", "double": "f8",
              "float64": "f8"}


def read_ply_vertices(path) -> dict[str, np.ndarray]:
    """The vertex properties of a binary PLY file (little or big endian, one vertex element
    with scalar properties, as 3DGS files are), by name."""
    data = Path(path).read_bytes()
    end = data.find(b"end_header")
    if not data.startswith(b"ply") or end < 0:
        raise ValueError(f"{path}: not a PLY file")
    body_start = data.index(b"\n", end) + 1
    header = data[:end].decode("ascii").splitlines()
    fmt, n, props, in_vertex = None, 0, [], False
    for line in header:
        tok = line.split()
        if not tok:
            continue
        if tok[0] == "format":
            fmt = tok[1]
        elif tok[0] == "element":
            in_vertex = tok[1] == "vertex"
            if in_vertex:
                n = int(tok[2])
            elif props or n:
                raise ValueError(f"{path}: only files whose first element is 'vertex' are read")
        elif tok[0] == "property" and in_vertex:
            if tok[1] == "list":
                raise ValueError(f"{path}: list properties are not supported")
            props.append((tok[2], _PLY_TYPES[tok[1]]))
    if fmt not in ("binary_little_endian", "binary_big_endian"):
        raise ValueError(f"{path}: unsupported PLY format {fmt!r}")
    order = "<" if fmt == "binary_little_endian" else ">"
    dt = np.dtype([(name, order + t) for name, t in props])
    rec = np.frombuffer(data, dtype=dt, count=n, offset=body_start)
    return {name: np.asarray(rec[name]) for name, _ in props}


def load_ply(path, device="cpu", max_sh_degree: int = 3) -> gaussian:
    """Reads an Inria-layout file back into a `gaussian` (the inverse of `save_ply`: log-scales,
    opacity logits, normalised quaternions, k_j [N, K, 3] from the channel-major f_rest)."""
    v = read_ply_vertices(path)
    n = int(v["x"].shape[0])
    n_rest = (max_sh_degree + 1) ** 2 - 1
    rest_names = sorted((k for k in v if k.startswith("f_rest_")), key=lambda k: int(k[7:]))
    f_rest = (np.stack([v[k] for k in rest_names], axis=1) if rest_names
              else np.zeros((n, 0), np.float32))
    k = f_rest.shape[1] // 3
    rest = f_rest.reshape(n, 3, k).transpose(0, 2, 1)  # (N, 3, K) -> (N, K, 3)
    if k < n_rest:
        rest = np.concatenate([rest, np.zeros((n, n_rest - k, 3), np.float32)], axis=1)
    g = gaussian(n)

    def col(*names):
        return torch.from_numpy(np.stack([v[name] for name in names], axis=1).astype(np.float32))

    g.mu = col("x", "y", "z").to(device).contiguous()
    g.A = col("f_dc_0", "f_dc_1", "f_dc_2").to(device).contiguous()
    g.k_j = torch.from_numpy(np.ascontiguousarray(rest[:, :n_rest], np.float32)).to(device)
    g.alpha = col("opacity").to(device).contiguous()
    g.s = col("scale_0", "scale_1", "scale_2").to(device).contiguous()
    g.q = col("rot_0", "rot_1", "rot_2", "rot_3").to(device).contiguous()
    return g
