"""The allocation-free pair-list entry point, s3dsp_kmap_pairs_noalloc.

Some callers cannot allocate device memory while they run — for example a
serving process that reserves its whole memory budget up front and hands the
library only pre-sized buffers, or code running where a cudaMalloc would
break its contract. For them the library offers a variant of
s3dsp_kmap_pairs whose scratch is a static device array (maps of at most
2^21 output rows). These tests call it through the C ABI and check that it
returns exactly what the allocating entry point returns, on two calls in a
row (the second call reuses the shared static scratch left by the first),
that it takes no memory from the library's pool (the allocating call does),
and that the largest accepted map works.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

import s3dsp
import workloads

pytestmark = pytest.mark.gpu

NOALLOC_MAX_ROWS = 1 << 21


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def build_kmap(ctx, coords):
    h = ctx.hash_build(torch.from_numpy(np.ascontiguousarray(coords)).cuda())
    return h, ctx.kmap_subm3(h)


def pairs_with(fn, ctx, kmap, n):
    cap = 27 * n
    pin = torch.full((cap,), -7, dtype=torch.int32, device="cuda")
    pout = torch.full((cap,), -7, dtype=torch.int32, device="cuda")
    offs = (ctypes.c_int64 * 28)()
    buf = ctypes.create_string_buffer(256)
    st = fn(ctx.handle, kmap.handle, pin.data_ptr(), pout.data_ptr(), cap, offs, buf, 256)
    assert st == s3dsp.S3D_OK, buf.value
    torch.cuda.synchronize()
    total = offs[27]
    return list(offs), pin[:total].cpu().numpy(), pout[:total].cpu().numpy()


def dense_block(side):
    g = np.arange(side, dtype=np.int32)
    x, y, z = np.meshgrid(g, g, g, indexing="ij")
    return np.stack([np.zeros_like(x), x, y, z], -1).reshape(-1, 4).astype(np.int32)


def test_noalloc_pairs_equal_allocating_pairs_twice_in_a_row(ctx):
    lib = s3dsp.load()
    shells = [workloads.ellipsoid_shell(64, 1), workloads.ellipsoid_shell(48, 2)]
    for coords in shells:  # two calls in a row, different maps
        _, k = build_kmap(ctx, coords)
        n = len(coords)
        ref_offs, ref_in, ref_out = pairs_with(lib.s3dsp_kmap_pairs, ctx, k, n)
        got_offs, got_in, got_out = pairs_with(lib.s3dsp_kmap_pairs_noalloc, ctx, k, n)
        assert got_offs == ref_offs
        assert ref_offs[27] > 0
        assert np.array_equal(got_in, ref_in)
        assert np.array_equal(got_out, ref_out)


def test_noalloc_takes_no_pool_memory(ctx):
    lib = s3dsp.load()
    coords = workloads.ellipsoid_shell(64, 3)
    _, k = build_kmap(ctx, coords)
    torch.cuda.synchronize()
    before = s3dsp.memory_stats(0, reset_high=True)
    pairs_with(lib.s3dsp_kmap_pairs_noalloc, ctx, k, len(coords))
    after = s3dsp.memory_stats(0)
    assert after["used_high"] == before["used"], (before, after)
    # the check is sensitive: the allocating call does take pool memory
    s3dsp.memory_stats(0, reset_high=True)
    pairs_with(lib.s3dsp_kmap_pairs, ctx, k, len(coords))
    assert s3dsp.memory_stats(0)["used_high"] > before["used"]


def test_noalloc_at_exactly_its_limit(ctx):
    # a dense 128^3 block has exactly 2^21 rows, the largest accepted map
    lib = s3dsp.load()
    coords = dense_block(128)
    assert len(coords) == NOALLOC_MAX_ROWS
    _, k = build_kmap(ctx, coords)
    ref_offs, ref_in, ref_out = pairs_with(lib.s3dsp_kmap_pairs, ctx, k, len(coords))
    got_offs, got_in, got_out = pairs_with(lib.s3dsp_kmap_pairs_noalloc, ctx, k, len(coords))
    assert got_offs == ref_offs
    # every interior voxel of the block has all 27 neighbours: 27 * 126^3 of them
    # plus the faces; the centre offset pairs every row with itself
    assert ref_offs[14] - ref_offs[13] == NOALLOC_MAX_ROWS
    assert np.array_equal(got_in, ref_in)
    assert np.array_equal(got_out, ref_out)


def test_noalloc_rejects_maps_above_its_limit(ctx):
    # eight voxels more than the dense 128^3 block
    extra = np.array([[0, 200, 0, j] for j in range(8)], np.int32)
    coords = np.concatenate([dense_block(128), extra]).astype(np.int32)
    assert len(coords) == NOALLOC_MAX_ROWS + 8
    _, k = build_kmap(ctx, coords)
    pin = torch.empty(16, dtype=torch.int32, device="cuda")
    pout = torch.empty(16, dtype=torch.int32, device="cuda")
    with pytest.raises(s3dsp.S3dError) as ei:
        ctx.kmap_pairs_noalloc(k, pin, pout)
    assert ei.value.status == s3dsp.S3D_INVALID_ARGUMENT
    assert "limited to 2097152 rows" in ei.value.message
