"""The coordinate pipeline on the device (s3dsp_occupancy_coords,
s3dsp_prune_surface, s3dsp_downsample_coords) against the oracle, bit-exact:
the reference's shipped SS occupancy fixture, a dense solid above the
downsample cap (the host-side random subsample), and the edge cases."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
from test_oracle_coords import fixture_grid

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def gpu_occ(ctx, grid, batch=0):
    g = torch.from_numpy(np.ascontiguousarray(grid, np.float32)).cuda()
    out = torch.empty((grid.size, 4), dtype=torch.int32, device="cuda")
    n = ctx.occupancy_coords(g, out, batch)
    return out[:n].cpu().numpy()


def gpu_prune(ctx, coords):
    d = torch.from_numpy(np.ascontiguousarray(coords)).cuda()
    out = torch.empty_like(d)
    n = ctx.prune_surface(d, out)
    return out[:n].cpu().numpy()


def gpu_down(ctx, coords, max_coords, seed=42):
    d = torch.from_numpy(np.ascontiguousarray(coords)).cuda()
    out = torch.empty_like(d)
    n = ctx.downsample_coords(d, out, max_coords, 2, seed)
    return out[:n].cpu().numpy()


def test_pipeline_on_ss_fixture(ctx, golden_dir):
    grid = fixture_grid(golden_dir)
    c = gpu_occ(ctx, grid)
    assert np.array_equal(c, oracle.occupancy_coords(grid))
    p = gpu_prune(ctx, c)
    assert np.array_equal(p, oracle.prune_surface(c))
    for cap, seed in ((42000, 42), (60000, 42), (5000, 42), (5000, 3)):
        assert np.array_equal(gpu_down(ctx, c, cap, seed), oracle.downsample_coords(c, cap, seed=seed)), (cap, seed)


def test_dense_solid_above_cap(ctx):
    # a solid ellipsoid: 502,712 cells, ~63k unique after halving
    ax = np.arange(128) + 0.5
    x, y, z = np.meshgrid(ax, ax, ax, indexing="ij")
    grid = (((x - 63) / 60) ** 2 + ((y - 60) / 50) ** 2 + ((z - 66) / 40) ** 2 <= 1.0).astype(np.float32)
    grid[grid > 0] = np.random.default_rng(0).uniform(0.1, 1.0, int(grid.sum()))
    c = gpu_occ(ctx, grid, batch=2)
    assert np.array_equal(c, oracle.occupancy_coords(grid, 2))
    p = gpu_prune(ctx, c)
    assert np.array_equal(p, oracle.prune_surface(c))
    for cap in (20000, 100000):  # halved (~63k unique) with and without the subsample
        assert np.array_equal(gpu_down(ctx, c, cap), oracle.downsample_coords(c, cap))


def test_edges(ctx):
    # empty grid, a grid too full for the output, a single voxel, negative coordinates
    assert len(gpu_occ(ctx, np.zeros((4, 5, 6), np.float32))) == 0
    g = torch.ones((4, 4, 4), device="cuda")
    small = torch.empty((10, 4), dtype=torch.int32, device="cuda")
    with pytest.raises(s3dsp.S3dError) as ei:
        ctx.occupancy_coords(g, small)
    assert ei.value.status == s3dsp.S3D_INVALID_ARGUMENT
    one = np.array([[0, 3, 4, 5]], np.int32)
    assert np.array_equal(gpu_prune(ctx, one), one)
    neg = np.array([[0, x, y, z] for x in range(-3, 2) for y in range(-2, 3) for z in range(-4, 1)], np.int32)
    assert np.array_equal(gpu_prune(ctx, neg), oracle.prune_surface(neg))
    assert np.array_equal(gpu_down(ctx, neg, 30), oracle.downsample_coords(neg, 30))
