"""The CPU oracle's integer tables, pinned to the reference.

Expected tables come from the reference's own SlatTables::build and
MeshSubdivideTables::build (src/objects_runtime/sparse_ops.cpp:49-173,
:272-404): committed goldens made by tests/golden/make_golden.py, and — when
oracle/_ref was built in this container — the compiled reference itself.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle
import workloads

TABLE_KEYS = ("fine_to_coarse", "coarse_children", "coarse_inv_count", "conv_fine", "conv_coarse")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).astype("<i4").tobytes()).hexdigest()


def sha_f(a):
    return hashlib.sha256(np.ascontiguousarray(a).astype("<f4").tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["kat_block3.npz", "shell16.npz"])
def test_oracle_matches_golden_full_tables(golden_dir, name):
    g = np.load(os.path.join(golden_dir, name))
    t = oracle.slat_tables(g["coords"])
    assert t["nc"] == int(g["nc"])
    for k in TABLE_KEYS:
        assert np.array_equal(t[k], g[k]), k
    cc, nb = oracle.mesh_subdivide(g["coords"])
    assert np.array_equal(cc, g["child_coords"])
    assert np.array_equal(nb, g["neighbors"])


def test_block3_known_answers(golden_dir):
    """Analytic checks on the full 3x3x3 block: the centre voxel sees all 27
    neighbours, a corner sees 8; one coarse cell per 2x2x2 parity class."""
    g = np.load(os.path.join(golden_dir, "kat_block3.npz"))
    coords = g["coords"]
    t = oracle.slat_tables(coords)
    conv = t["conv_fine"].reshape(-1, 27)
    centre = int(np.nonzero((coords[:, 1:] == 31).all(1))[0][0])
    assert (conv[centre] < 27).sum() == 27
    assert np.array_equal(conv[centre], np.arange(27))  # lexicographic block: offset o -> row o
    corner = int(np.nonzero((coords[:, 1:] == 30).all(1))[0][0])
    assert (conv[corner] < 27).sum() == 8
    # x,y,z in {30,31,32} -> x//2 in {15,16}: 8 coarse cells
    assert t["nc"] == 8
    # mesh: 216 children, child 0 of parent 0 is (60,60,60)
    cc, nb = oracle.mesh_subdivide(coords)
    assert cc.shape == (216, 4) and tuple(cc[0]) == (0, 60, 60, 60)
    assert (nb >= 0).sum(1).max() == 27


def test_oracle_edge_cases(golden_dir):
    g = np.load(os.path.join(golden_dir, "edge_cases.npz"))
    for name in ("multi", "multi_unique", "dup_rows"):
        t = oracle.slat_tables(g[name + "_coords"])
        assert t["nc"] == int(g[name + "_nc"]), name
        for k in TABLE_KEYS:
            assert np.array_equal(t[k], g[f"{name}_{k}"]), (name, k)
        m = oracle.mesh_subdivide(g[name + "_coords"])
        assert (m is not None) == bool(g[name + "_mesh_ok"]), name
        if m is not None:
            assert np.array_equal(m[0], g[name + "_child_coords"])
            assert np.array_equal(m[1], g[name + "_neighbors"])


def test_oracle_matches_golden_digests(golden_dir):
    with open(os.path.join(golden_dir, "digests.json")) as f:
        d = json.load(f)
    shell = workloads.ellipsoid_shell(64, 0)
    e = d["config1_shell"]
    assert len(shell) == e["n"] and sha(shell) == e["coords"]
    t = oracle.slat_tables(shell)
    assert t["nc"] == e["nc"]
    for k in ("conv_fine", "conv_coarse", "fine_to_coarse", "coarse_children"):
        assert sha(t[k]) == e[k], k
    assert sha_f(t["coarse_inv_count"]) == e["coarse_inv_count"]
    cc, nb = oracle.mesh_subdivide(shell)
    assert sha(cc) == e["child_coords"] and sha(nb) == e["neighbors"]
    e2 = d["config1_subdivide2"]
    cc2, nb2 = oracle.mesh_subdivide(cc)
    assert len(cc) == e2["n"] and sha(cc2) == e2["child_coords"] and sha(nb2) == e2["neighbors"]


def ss_occ_pruned(golden_dir):
    bits = np.load(os.path.join(golden_dir, "ss_occ_mask.npz"))["bits"]
    mask = np.unpackbits(bits)[: 64 ** 3].astype(bool).reshape(64, 64, 64)
    x, y, z = np.nonzero(mask)
    occ = np.stack([np.zeros_like(x), x, y, z], 1).astype(np.int32)
    pad = np.zeros((66, 66, 66), bool)
    pad[occ[:, 1] + 1, occ[:, 2] + 1, occ[:, 3] + 1] = True
    keep = np.zeros(len(occ), bool)
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                keep |= ~pad[occ[:, 1] + 1 + dx, occ[:, 2] + 1 + dy, occ[:, 3] + 1 + dz]
    return occ, occ[keep]


def test_oracle_real_occupancy_fixture(golden_dir):
    """The reference's shipped 64^3 SS-decoder occupancy (69,537 occupied,
    67,783 after surface pruning) as a realistic hash / kmap stress set."""
    with open(os.path.join(golden_dir, "digests.json")) as f:
        e = json.load(f)["ss_occ_pruned"]
    occ, pruned = ss_occ_pruned(golden_dir)
    assert len(occ) == e["n_occupied"] and len(pruned) == e["n"] and sha(pruned) == e["coords"]
    t = oracle.slat_tables(pruned)
    assert t["nc"] == e["nc"]
    for k in ("conv_fine", "conv_coarse", "fine_to_coarse", "coarse_children"):
        assert sha(t[k]) == e[k], k
    cc, nb = oracle.mesh_subdivide(pruned)
    assert sha(cc) == e["child_coords"] and sha(nb) == e["neighbors"]


def test_oracle_rejects_like_reference():
    assert oracle.slat_tables(np.zeros((0, 4), np.int32)) is None          # sparse_ops.cpp:51
    assert oracle.mesh_subdivide(np.zeros((0, 4), np.int32)) is None       # :273
    dup = np.array([[0, 1, 2, 3], [0, 1, 2, 3]], np.int32)
    assert oracle.mesh_subdivide(dup) is None                              # :325-333


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built in this container")
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_matches_compiled_reference(seed):
    rng = np.random.default_rng(seed)
    shell = workloads.ellipsoid_shell(32, seed)
    # shuffle rows, add a second batch and negative coordinates
    other = shell.copy()
    other[:, 0] = 3
    other[:, 1:] -= 20
    coords = np.concatenate([shell, other])[rng.permutation(2 * len(shell))]
    a = oracle.slat_tables(coords)
    b = oracle.slat_tables(coords, use_ref=True)
    assert a["nc"] == b["nc"]
    for k in TABLE_KEYS:
        assert np.array_equal(a[k], b[k]), k
    ma, mb = oracle.mesh_subdivide(coords), oracle.mesh_subdivide(coords, use_ref=True)
    assert np.array_equal(ma[0], mb[0]) and np.array_equal(ma[1], mb[1])


def gs_cases():
    rng = np.random.default_rng(3)
    shell = workloads.ellipsoid_shell(64, 0)
    multi = np.concatenate([workloads.ellipsoid_shell(32, 1, batch=0), workloads.ellipsoid_shell(32, 2, batch=1)])
    neg = np.array([[0, x, y, z] for x in range(-9, 3) for y in range(-5, 7) for z in range(-12, 1)], np.int32)
    return {"shell64": shell, "shell64_shuffled": shell[rng.permutation(len(shell))],
            "multi_batch_shuffled": multi[rng.permutation(len(multi))], "negative": neg,
            "one": np.array([[0, 5, 6, 7]], np.int32)}


@pytest.mark.skipif(not oracle.ref_available(), reason="reference table builder not built")
@pytest.mark.parametrize("name", list(gs_cases()))
def test_oracle_gs_tables_match_reference(name):
    """The restated GsTables::build (window buckets for both shifts, APE) equals
    the reference's own, compiled from sparse_ops.cpp."""
    coords = gs_cases()[name]
    for si in (0, 1):
        mine = oracle.gs_window_tables(coords, si)
        ref = oracle.gs_window_tables(coords, si, use_ref=True)
        for a, b in zip(mine, ref):
            assert np.array_equal(a, b), (name, si)
    assert np.array_equal(oracle.ape(coords), oracle.ape(coords, use_ref=True))
