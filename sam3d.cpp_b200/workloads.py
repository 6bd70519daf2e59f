"""Seeded synthetic inputs for the sparse-convolution path.

The reference measures on a real object (about 27k active voxels at 64^3 after
surface pruning, sam3d.cpp reference/OBJECTS_RUNTIME.md:75-76); these
generators stand in for it with ellipsoid shells of the same size and
value distributions. Every generator is a pure function of its seed, so the
CPU oracle and the GPU path see identical bytes.

Coordinates are int32 rows (batch, x, y, z) in lexicographic (x, y, z) order,
the order in which the reference extracts occupied cells from the SS decoder
occupancy grid (src/objects_runtime/session.cpp:1436-1441).
"""
from __future__ import annotations

import numpy as np


def ellipsoid_shell(res: int = 64, seed: int = 0, thickness: float = 1.5,
                    axes_range=(16.0, 30.0), centre_jitter: float = 4.0,
                    batch: int = 0) -> np.ndarray:
    """Voxels whose centre lies within +-thickness voxels of an ellipsoid surface.

    Semi-axes a ~ U[axes_range]^3 and centre c = res/2 + U[-jitter, jitter]^3,
    both scaled by res/64 so that larger grids hold the same shape. A voxel
    (i, j, k) with centre p = (i, j, k) + 0.5 is kept when
    | |p - c| * (1 - 1/|(p - c) / a|) | <= thickness, i.e. its radial distance
    to the surface along the ray from the centre is at most `thickness`.
    Returns int32 [N, 4] coords (batch, x, y, z), lexicographically sorted.
    """
    rng = np.random.default_rng(seed)
    scale = res / 64.0
    a = rng.uniform(axes_range[0], axes_range[1], size=3) * scale
    c = res / 2.0 + rng.uniform(-centre_jitter, centre_jitter, size=3) * scale
    keep = []
    ax = np.arange(res, dtype=np.float64) + 0.5
    # process one x-slab at a time to bound memory at large res
    gy, gz = np.meshgrid(ax, ax, indexing="ij")
    for i in range(res):
        d = np.stack([np.full_like(gy, ax[i]) - c[0], gy - c[1], gz - c[2]], axis=-1)
        r = np.sqrt((d * d).sum(-1))
        q = np.sqrt(((d / a) ** 2).sum(-1))
        with np.errstate(divide="ignore", invalid="ignore"):
            dist = np.abs(r * (1.0 - 1.0 / q))
        dist[q == 0] = np.inf
        jj, kk = np.nonzero(dist <= thickness)
        if len(jj):
            keep.append(np.stack([np.full_like(jj, batch), np.full_like(jj, i), jj, kk], axis=1))
    coords = np.concatenate(keep, axis=0).astype(np.int32)
    return np.ascontiguousarray(coords)


def ellipsoid_shell_device(res: int = 64, seed: int = 0, thickness: float = 1.5,
                           axes_range=(16.0, 30.0), centre_jitter: float = 4.0, batch: int = 0,
                           device="cuda") -> np.ndarray:
    """`ellipsoid_shell` evaluated with torch on `device` (for large grids: the
    512^3 volume takes seconds in numpy). Identical output: the same seeded
    draws on the host, then the same IEEE float64 operations in the same
    order (products, sums left to right, correctly rounded divide and square
    root; no fused multiply-add), and the kept voxels in lexicographic order.
    Returns int32 [N, 4] on the host."""
    import torch

    rng = np.random.default_rng(seed)
    scale = res / 64.0
    a = rng.uniform(axes_range[0], axes_range[1], size=3) * scale
    c = res / 2.0 + rng.uniform(-centre_jitter, centre_jitter, size=3) * scale
    ax = torch.arange(res, dtype=torch.float64, device=device) + 0.5
    dy = (ax - float(c[1])).view(1, -1, 1)
    dz = (ax - float(c[2])).view(1, 1, -1)
    qy, qz = dy / float(a[1]), dz / float(a[2])
    out = []
    chunk = max(1, (1 << 24) // (res * res))  # x-slabs per pass, ~16M voxels
    for i0 in range(0, res, chunk):
        dx = (ax[i0:i0 + chunk] - float(c[0])).view(-1, 1, 1)
        qx = dx / float(a[0])
        r = torch.sqrt(dx * dx + dy * dy + dz * dz)
        q = torch.sqrt(qx * qx + qy * qy + qz * qz)
        dist = torch.abs(r * (1.0 - 1.0 / q))
        dist = torch.where(q == 0, torch.full_like(dist, float("inf")), dist)
        idx = torch.nonzero(dist <= thickness)
        idx[:, 0] += i0
        out.append(idx)
    ijk = torch.cat(out).to(torch.int32).cpu().numpy()
    coords = np.empty((len(ijk), 4), np.int32)
    coords[:, 0] = batch
    coords[:, 1:] = ijk
    return np.ascontiguousarray(coords)


def normal(shape, seed: int, std: float = 1.0) -> np.ndarray:
    """float32 N(0, std^2) with a numpy default_rng seed."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(size=shape) * std).astype(np.float32)


def conv_weight_slat(cin: int, cout: int, seed: int, std: float | None = None) -> np.ndarray:
    """SubMConv3d weight in the SLat GGUF row layout (Cout, 27*Cin), i.e. the
    spconv checkpoint (Cout, 3, 3, 3, Cin) flattened
    (scripts/objects/gguf_schema.py:326-334). Default std = sqrt(1/(27*Cin))."""
    if std is None:
        std = float(np.sqrt(1.0 / (27 * cin)))
    return normal((cout, 27 * cin), seed, std)


def kaiming_normal_slat(cin: int, cout: int, seed: int) -> np.ndarray:
    """Kaiming-normal (fan_in = 27*Cin, gain sqrt(2)) in the SLat row layout."""
    return conv_weight_slat(cin, cout, seed, std=float(np.sqrt(2.0 / (27 * cin))))


def slat_to_mesh_packed(w_slat: np.ndarray, cin: int, cout: int) -> np.ndarray:
    """(Cout, 27*Cin) -> (27, Cout*Cin): the mesh decoder's packed layout
    (scripts/objects/convert_sam3d_to_gguf.py:481-492, permute(1,2,3,0,4))."""
    return np.ascontiguousarray(
        w_slat.reshape(cout, 27, cin).transpose(1, 0, 2).reshape(27, cout * cin))


def config1(seed: int = 0):
    """Config 1: one subm conv, 64^3 shell (~20k voxels), Cin = Cout = 64.
    Features N(0,1), W ~ N(0, 1/(27*Cin)), bias ~ N(0, 0.01)."""
    coords = ellipsoid_shell(64, seed)
    n = len(coords)
    return dict(coords=coords, feats=normal((n, 64), seed + 1),
                weight=conv_weight_slat(64, 64, seed + 2),
                bias=normal((64,), seed + 3, std=0.1), cin=64, cout=64)


def config2(seed: int = 0, channels: int = 256):
    """Config 2: residual block on the config-1 shell, C = 256:
    subm conv3 -> GroupNorm(32) -> SiLU -> subm conv3 -> + skip.
    Kaiming-normal weights, gamma = 1, beta = 0, biases N(0, 0.01)."""
    coords = ellipsoid_shell(64, seed)
    n = len(coords)
    c = channels
    return dict(coords=coords, feats=normal((n, c), seed + 1),
                w1=kaiming_normal_slat(c, c, seed + 2), b1=normal((c,), seed + 3, std=0.1),
                gamma=np.ones(c, np.float32), beta=np.zeros(c, np.float32),
                w2=kaiming_normal_slat(c, c, seed + 4), b2=normal((c,), seed + 5, std=0.1),
                channels=c, groups=32)


def config3(seed: int = 1, cin: int = 128, cout: int = 64):
    """Config 3: stride-2 subdivide of the config-1 shell (every parent spawns
    its 8 children, ~160k outputs) as a learned 2x2x2 transposed conv
    Cin -> Cout, then one subm conv3 at Cout. Features N(0,1)."""
    coords = ellipsoid_shell(64, 0)
    n = len(coords)
    return dict(coords=coords, feats=normal((n, cin), seed + 1),
                w_up=normal((8, cout, cin), seed + 2, std=float(np.sqrt(1.0 / cin))),
                b_up=normal((cout,), seed + 3, std=0.1),
                w=conv_weight_slat(cout, cout, seed + 4), b=normal((cout,), seed + 5, std=0.1),
                cin=cin, cout=cout)


def ellipsoid_params(res: int = 64, seed: int = 0, axes_range=(16.0, 30.0), centre_jitter: float = 4.0):
    """The semi-axes and centre `ellipsoid_shell(res, seed)` draws."""
    rng = np.random.default_rng(seed)
    scale = res / 64.0
    a = rng.uniform(axes_range[0], axes_range[1], size=3) * scale
    c = res / 2.0 + rng.uniform(-centre_jitter, centre_jitter, size=3) * scale
    return a, c


MESH_RES = 256
MESH_RAW = 101


def subdivide_order(parents: np.ndarray, levels: int = 2) -> np.ndarray:
    """Children of `parents` after `levels` stride-2 subdivisions, in the
    mesh decoder's row order (parent-major, child j = xb*4 + yb*2 + zb)."""
    c = np.asarray(parents, np.int32)
    off = np.array([[0, (j >> 2) & 1, (j >> 1) & 1, j & 1] for j in range(8)], np.int32)
    scale = np.array([1, 2, 2, 2], np.int32)
    for _ in range(levels):
        c = (c[:, None, :] * scale + off[None]).reshape(-1, 4)
    return np.ascontiguousarray(c)


def flexicubes_input(parent_res: int = 64, seed: int = 0, sdf_noise: float = 0.3, thickness: float = 1.5):
    """Stand-in for the mesh decoder's final output at 256^3: the cubes of the
    config-1-style shell at `parent_res` after two subdivisions (x4 per axis,
    mesh decoder row order) and raw [N, 101] features in the extractor's
    channel layout: 0-7 corner SDFs, 8-31 corner deformations, 32-52
    FlexiCubes weights, 53-100 corner colours.

    The corner SDFs are the signed radial distance of the corner to the
    ellipsoid surface in grid units of 1/256, plus the extractor's 1/256
    offset, plus N(0, sdf_noise/256) noise so that ambiguous cube
    configurations occur; the other channels are N(0, 0.5^2) / N(0, 1)."""
    assert parent_res * 4 <= MESH_RES
    parents = ellipsoid_shell(parent_res, seed, thickness=thickness)
    cubes = subdivide_order(parents, 2)
    n = len(cubes)
    a, c = ellipsoid_params(parent_res, seed)
    a, c = a * 4.0, c * 4.0
    corners = np.array([[0, 0, 0], [1, 0, 0], [0, 1, 0], [1, 1, 0], [0, 0, 1], [1, 0, 1], [0, 1, 1], [1, 1, 1]],
                       np.float64)
    p = cubes[:, None, 1:].astype(np.float64) + corners[None]  # [n, 8, 3]
    d = p - c
    r = np.sqrt((d * d).sum(-1))
    q = np.sqrt(((d / a) ** 2).sum(-1))
    with np.errstate(divide="ignore", invalid="ignore"):
        dist = np.where(q > 0, r * (1.0 - 1.0 / q), -1.0)
    rng = np.random.default_rng(seed + 17)
    raw = np.empty((n, MESH_RAW), np.float32)
    raw[:, 0:8] = (dist + 1.0 + rng.normal(0.0, sdf_noise, size=(n, 8))) / MESH_RES
    raw[:, 8:32] = rng.normal(0.0, 0.5, size=(n, 24))
    raw[:, 32:53] = rng.normal(0.0, 1.0, size=(n, 21))
    raw[:, 53:101] = rng.normal(0.0, 1.0, size=(n, 48))
    return cubes, raw
