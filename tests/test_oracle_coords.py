"""Oracle restatement of the coordinate pipeline (session.cpp argwhere,
prune_surface_coords, downsample_coords) on CPU: the reference's shipped SS
occupancy fixture reproduces its recorded counts and digest, and downsample
keeps its invariants."""
import hashlib
import json
import os

import numpy as np

import oracle
from test_oracle_tables import ss_occ_pruned


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def fixture_grid(golden_dir):
    bits = np.load(os.path.join(golden_dir, "ss_occ_mask.npz"))["bits"]
    return np.unpackbits(bits)[: 64 ** 3].astype(np.float32).reshape(64, 64, 64)


def test_argwhere_and_prune_on_fixture(golden_dir):
    with open(os.path.join(golden_dir, "digests.json")) as f:
        e = json.load(f)["ss_occ_pruned"]
    occ, pruned = ss_occ_pruned(golden_dir)
    c = oracle.occupancy_coords(fixture_grid(golden_dir))
    assert len(c) == e["n_occupied"] and np.array_equal(c, occ)
    p = oracle.prune_surface(c)
    assert len(p) == e["n"] and sha(p) == e["coords"] and np.array_equal(p, pruned)


def test_downsample_invariants(golden_dir):
    c = oracle.occupancy_coords(fixture_grid(golden_dir))
    assert np.array_equal(oracle.downsample_coords(c, len(c)), c)  # at or under the cap: unchanged
    d = oracle.downsample_coords(c, 42000)
    assert len(d) < len(c)
    assert len({tuple(r) for r in d.tolist()}) == len(d)  # first occurrences only
    lo, hi = c[:, 1:].min(0), c[:, 1:].max(0)
    ext = hi - lo + 1
    assert np.all(d[:, 1:].max(0) - d[:, 1:].min(0) + 1 <= (ext + 1) // 2 + 1)
    s = oracle.downsample_coords(c, 5000, seed=7)
    assert len(s) == 5000
    assert {tuple(r) for r in s.tolist()} <= {tuple(r) for r in d.tolist()}
    assert np.array_equal(s, oracle.downsample_coords(c, 5000, seed=7))
    assert not np.array_equal(s, oracle.downsample_coords(c, 5000, seed=8))
