"""The FlexiCubes restatement (oracle/s3d_oracle.cpp, mesh_extractor.cpp:95-377)
against the reference: its committed outputs and digests, and, where the
reference's extractor is compiled into oracle/_ref, the reference itself."""
import hashlib

import numpy as np
import pytest

import oracle
import workloads
from flexicubes_check import GOLDEN, boundary_random, digests, single_cube, tables


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).astype("<i4").tobytes()).hexdigest()


def test_small_fixture_exact():
    g = np.load(GOLDEN + "/flexicubes_small.npz")
    c, r = workloads.flexicubes_input(int(g["parent_res"]), int(g["seed"]))
    assert len(c) == int(g["n"])
    m = oracle.flexicubes(r, c, tables())
    for k in ("vertices", "attrs", "faces", "surface", "cases", "edges"):
        assert np.array_equal(m[k], g[k]), k


@pytest.mark.parametrize("name", ["flexicubes_noisy16", "flexicubes_full64"])
def test_topology_digests(name):
    d = digests()[name]
    kw = {k: d[k] for k in ("parent_res", "seed", "sdf_noise") if k in d}
    c, r = workloads.flexicubes_input(**kw)
    assert len(c) == d["n"]
    m = oracle.flexicubes(r, c, tables())
    for k in ("faces", "surface", "cases", "edges"):
        assert sha(m[k]) == d[k], k
    assert len(m["vertices"]) == d["n_vertices"]


@pytest.mark.parametrize("bad,msg", [
    (np.array([[0, 1, 2, 3], [1, 0, 0, 0]], np.int32), "batch one"),
    (np.array([[0, 1, 2, 3], [0, 0, 256, 0]], np.int32), "outside resolution 256"),
    (np.array([[0, 1, 2, 3], [0, 0, -1, 0]], np.int32), "outside resolution 256"),
    (np.array([[0, 1, 2, 3], [0, 4, 4, 4], [0, 1, 2, 3]], np.int32), "duplicate"),
    # the first offending row decides the message
    (np.array([[0, 1, 2, 3], [0, 1, 2, 3], [2, 0, 0, 0]], np.int32), "duplicate"),
    (np.array([[0, 1, 2, 3], [0, 300, 0, 0], [0, 1, 2, 3]], np.int32), "outside resolution 256"),
])
def test_input_errors(bad, msg):
    with pytest.raises(ValueError, match=msg):
        oracle.flexicubes(np.zeros((len(bad), 101), np.float32), bad, tables())


@pytest.mark.skipif(not oracle.ref_available(), reason="reference extractor not built")
def test_tables_fixture_is_the_reference_tables():
    t, f = oracle.ref_flexicubes_tables(), tables()
    for k in t:
        assert np.array_equal(t[k], f[k]), k


@pytest.mark.skipif(not oracle.ref_available(), reason="reference extractor not built")
@pytest.mark.parametrize("case", ["boundary_random", "single_cube", "shuffled_rows"])
def test_matches_reference(case):
    if case == "boundary_random":
        c, r = boundary_random()
    elif case == "single_cube":
        c, r = single_cube()
    else:
        c, r = workloads.flexicubes_input(8, 2, sdf_noise=1.0)
        p = np.random.default_rng(0).permutation(len(c))
        c, r = np.ascontiguousarray(c[p]), np.ascontiguousarray(r[p])
    a = oracle.flexicubes(r, c, tables())
    b = oracle.flexicubes(r, c, use_ref=True)
    for k in a:
        assert np.array_equal(a[k], b[k]), k
