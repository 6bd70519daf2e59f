"""Shared inputs and mesh comparison for the FlexiCubes extraction tests
(extract_object_mesh, src/objects_runtime/mesh_extractor.cpp:95-377)."""
import json
import os

import numpy as np

import workloads

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# float outputs pass through tanhf / expf (CUDA vs the host's libm): a few ulps
VERTEX_ABS_TOL = 1e-5


def tables():
    t = np.load(os.path.join(GOLDEN, "flexicubes_tables.npz"))
    return dict(dmc=t["dmc"], num_dual=t["num_dual"], check=t["check"])


def digests():
    with open(os.path.join(GOLDEN, "digests.json")) as f:
        return json.load(f)


def boundary_random(seed=5):
    """Random cubes in two corners of the grid (coordinates 0..5 and
    250..255), shuffled, with small random SDFs: grid-boundary edges, cubes
    without an input row, ambiguous cases."""
    rng = np.random.default_rng(seed)
    pts = np.concatenate([rng.integers(0, 6, (3000, 3)), rng.integers(250, 256, (3000, 3))])
    pts = np.unique(pts, axis=0).astype(np.int32)
    c = np.concatenate([np.zeros((len(pts), 1), np.int32), pts], 1)[rng.permutation(len(pts))]
    raw = rng.normal(0, 1, (len(c), 101)).astype(np.float32)
    raw[:, :8] *= 0.01
    return np.ascontiguousarray(c), raw


def single_cube(seed=9):
    rng = np.random.default_rng(seed)
    return np.array([[0, 10, 20, 30]], np.int32), rng.normal(0, 1, (1, 101)).astype(np.float32)


def cases():
    """name -> (coords, raw)."""
    out = {}
    c, r = workloads.flexicubes_input(8, 0)
    out["small8"] = (c, r)
    c, r = workloads.flexicubes_input(16, 1, sdf_noise=3.0)
    out["noisy16"] = (c, r)
    out["boundary_random"] = boundary_random()
    out["single_cube"] = single_cube()
    return out


def dual_gamma64(mesh, coords, raw, tab):
    """float64 gamma of every dual vertex, from the dual numbering (dual
    count, surface order, local index) and the cube's input row."""
    nd = tab["num_dual"][mesh["cases"]].astype(np.int64)
    ids = (coords[:, 1].astype(np.int64) * 256 + coords[:, 2]) * 256 + coords[:, 3]
    order = np.argsort(ids)
    pos = np.searchsorted(ids[order], mesh["surface"])
    pos = np.minimum(pos, len(ids) - 1)
    hit = ids[order][pos] == mesh["surface"]
    rows = np.where(hit, order[pos], -1)
    w = np.where(rows >= 0, raw[np.maximum(rows, 0), 52].astype(np.float64), 0.0)
    g = 1.0 / (1.0 + np.exp(-w)) * 0.99 + 0.005
    return np.concatenate([np.repeat(g[nd == k], k) for k in (1, 2, 3, 4)])


def compare(got, exp, coords, raw, tab):
    """Topology identical; positions / attributes within VERTEX_ABS_TOL; a
    quad may take the other diagonal only when its gamma products tie to
    1e-5 relative (an ulp-level difference of expf decides such a split)."""
    for k in ("surface", "cases", "edges"):
        assert got[k].shape == exp[k].shape, k
        assert np.array_equal(got[k], exp[k]), k
    assert got["vertices"].shape == exp["vertices"].shape
    assert np.abs(got["vertices"] - exp["vertices"]).max(initial=0) <= VERTEX_ABS_TOL
    assert np.abs(got["attrs"] - exp["attrs"]).max(initial=0) <= VERTEX_ABS_TOL
    assert got["faces"].shape == exp["faces"].shape
    gq = got["faces"].reshape(-1, 6)
    eq = exp["faces"].reshape(-1, 6)
    bad = np.nonzero((gq != eq).any(1))[0]
    if len(bad):
        g = dual_gamma64(exp, coords, raw, tab)
        for q in bad:
            assert sorted(set(gq[q])) == sorted(set(eq[q])), f"quad {q} differs in its vertices"
            o = eq[q][[0, 1, 2, 5]]  # (o0, o1, o2, o3) for either split
            if eq[q][2] == eq[q][3]:  # split 2 writes o0, o1, o3, o3, o1, o2
                o = eq[q][[0, 1, 5, 2]]
            a, b = g[o[0]] * g[o[2]], g[o[1]] * g[o[3]]
            assert abs(a - b) <= 1e-5 * max(a, b), f"quad {q}: split differs away from a tie"
    return len(bad)
