"""Coordinate hash and kernel maps on the GPU, bit-exact against the reference tables.

Expected tables: the oracle restatement (itself pinned to the reference's
sparse_ops.cpp by test_oracle_tables.py) and the committed golden digests made
by the reference's own builders.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads

pytestmark = pytest.mark.gpu


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).astype("<i4").tobytes()).hexdigest()


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gpu_subm_tables(ctx, coords):
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    n = len(coords)
    out_slat = torch.empty((n, 27), dtype=torch.int32, device="cuda")
    out_mesh = torch.empty((n, 27), dtype=torch.int32, device="cuda")
    ctx.kmap_export_dense(k, s3dsp.SENTINEL_SLAT_N, out_slat)
    ctx.kmap_export_dense(k, s3dsp.SENTINEL_MESH_NEG1, out_mesh)
    torch.cuda.synchronize()
    return out_slat.cpu().numpy(), out_mesh.cpu().numpy(), h, k


def gpu_subdivide(ctx, parents):
    h = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(h, cc)
    nb = torch.empty((8 * len(parents), 27), dtype=torch.int32, device="cuda")
    ctx.kmap_export_dense(k, s3dsp.SENTINEL_MESH_NEG1, nb)
    torch.cuda.synchronize()
    return cc.cpu().numpy(), nb.cpu().numpy(), k


@pytest.mark.parametrize("seed,res", [(0, 64), (1, 64), (3, 16), (4, 128)])
def test_subm_kmap_bit_exact(ctx, seed, res):
    coords = workloads.ellipsoid_shell(res, seed)
    slat, mesh, _, _ = gpu_subm_tables(ctx, coords)
    t = oracle.slat_tables(coords)
    exp = t["conv_fine"].reshape(-1, 27)
    assert np.array_equal(slat, exp)
    assert np.array_equal(mesh, np.where(exp >= len(coords), -1, exp))


def test_subm_kmap_large_table_with_duplicates(ctx):
    """Above 16 MB of hash table (> 262k rows) the map reads each row's first
    row from the hash's self-row pass: 968k shell voxels plus 5,000 repeated
    rows, shuffled, must still match the reference table builder's rules."""
    base = workloads.ellipsoid_shell(512, 0)
    rng = np.random.default_rng(9)
    coords = np.concatenate([base, base[rng.choice(len(base), 5000, replace=False)]])
    coords = np.ascontiguousarray(coords[rng.permutation(len(coords))])
    slat, _, _, _ = gpu_subm_tables(ctx, coords)
    exp = oracle.slat_tables(coords)["conv_fine"].reshape(-1, 27)
    assert np.array_equal(slat, exp)


def test_subm_kmap_golden_digest(ctx, golden_dir):
    with open(os.path.join(golden_dir, "digests.json")) as f:
        e = json.load(f)["config1_shell"]
    coords = workloads.ellipsoid_shell(64, 0)
    slat, _, _, _ = gpu_subm_tables(ctx, coords)
    assert sha(slat.reshape(-1)) == e["conv_fine"]


def test_subm_kmap_duplicates_multibatch_negative(ctx, golden_dir):
    g = np.load(os.path.join(golden_dir, "edge_cases.npz"))
    for name in ("multi", "multi_unique", "dup_rows"):
        coords = g[name + "_coords"]
        slat, _, _, _ = gpu_subm_tables(ctx, coords)
        assert np.array_equal(slat.reshape(-1), g[name + "_conv_fine"]), name


def test_real_occupancy_fixture(ctx, golden_dir):
    from test_oracle_tables import ss_occ_pruned
    with open(os.path.join(golden_dir, "digests.json")) as f:
        e = json.load(f)["ss_occ_pruned"]
    _, pruned = ss_occ_pruned(golden_dir)
    slat, _, _, _ = gpu_subm_tables(ctx, pruned)
    assert sha(slat.reshape(-1)) == e["conv_fine"]
    cc, nb, _ = gpu_subdivide(ctx, pruned)
    assert sha(cc) == e["child_coords"] and sha(nb) == e["neighbors"]


@pytest.mark.parametrize("name", ["kat_block3.npz", "shell16.npz"])
def test_subdivide_golden_full(ctx, golden_dir, name):
    g = np.load(os.path.join(golden_dir, name))
    cc, nb, _ = gpu_subdivide(ctx, g["coords"])
    assert np.array_equal(cc, g["child_coords"])
    assert np.array_equal(nb, g["neighbors"])


def test_subdivide_two_levels_digest(ctx, golden_dir):
    with open(os.path.join(golden_dir, "digests.json")) as f:
        d = json.load(f)
    coords = workloads.ellipsoid_shell(64, 0)
    cc, nb, _ = gpu_subdivide(ctx, coords)
    assert sha(cc) == d["config1_shell"]["child_coords"] and sha(nb) == d["config1_shell"]["neighbors"]
    cc2, nb2, _ = gpu_subdivide(ctx, cc)
    assert sha(cc2) == d["config1_subdivide2"]["child_coords"]
    assert sha(nb2) == d["config1_subdivide2"]["neighbors"]


def test_subdivide_rejects_duplicates(ctx):
    dup = np.array([[0, 1, 2, 3], [0, 4, 5, 6], [0, 1, 2, 3]], np.int32)
    with pytest.raises(s3dsp.S3dError) as ei:
        ctx.hash_build(dev(dup), reject_duplicates=True)
    assert ei.value.status == s3dsp.S3D_INVALID_ARGUMENT


def test_hash_rejects_out_of_domain(ctx):
    bad = np.array([[0, 1, 2, 3], [0, 40000, 0, 0]], np.int32)
    with pytest.raises(s3dsp.S3dError):
        ctx.hash_build(dev(bad))
    with pytest.raises(s3dsp.S3dError):
        ctx.hash_build(dev(np.zeros((0, 4), np.int32)))


def test_hash_lookup(ctx):
    coords = workloads.ellipsoid_shell(32, 2)
    h = ctx.hash_build(dev(coords))
    q = np.concatenate([coords[::7], coords[::11] + np.array([0, 100, 0, 0], np.int32)])
    rows = torch.empty(len(q), dtype=torch.int32, device="cuda")
    ctx.hash_lookup(h, dev(q), rows)
    got = rows.cpu().numpy()
    n7 = len(coords[::7])
    assert np.array_equal(got[:n7], np.arange(0, len(coords), 7))
    assert (got[n7:] == -1).all()


def test_pairs_offset_sorted(ctx):
    coords = workloads.ellipsoid_shell(64, 1)
    slat, mesh, h, k = gpu_subm_tables(ctx, coords)
    n = len(coords)
    cap = 27 * n
    pin = torch.empty(cap, dtype=torch.int32, device="cuda")
    pout = torch.empty(cap, dtype=torch.int32, device="cuda")
    offs = ctx.kmap_pairs(k, pin, pout)
    pin, pout = pin.cpu().numpy(), pout.cpu().numpy()
    assert offs[0] == 0 and offs[27] == (mesh >= 0).sum()
    for o in range(27):
        rows = np.nonzero(mesh[:, o] >= 0)[0]
        seg = slice(offs[o], offs[o + 1])
        assert np.array_equal(pout[seg], rows)
        assert np.array_equal(pin[seg], mesh[rows, o])
