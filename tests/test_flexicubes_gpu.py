"""FlexiCubes extraction on the device (s3dsp_flexicubes_extract) against the
oracle restatement, itself pinned to the reference's extract_object_mesh:
topology identical, positions / attributes within a few ulps, and the
full-size topology against the reference's own digests."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from flexicubes_check import cases, compare, digests, tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


@pytest.fixture(scope="module")
def dtab(ctx):
    t = tables()
    return ctx.flexicubes_tables(t["dmc"], t["num_dual"], t["check"])


def run(ctx, dtab, coords, raw):
    m = ctx.flexicubes(dtab, torch.from_numpy(raw).cuda(), torch.from_numpy(coords).cuda())
    try:
        return m.host()
    finally:
        m.free()


@pytest.mark.parametrize("name", list(cases()))
def test_matches_oracle(ctx, dtab, name):
    coords, raw = cases()[name]
    got = run(ctx, dtab, coords, raw)
    exp = oracle.flexicubes(raw, coords, tables())
    compare(got, exp, coords, raw, tables())


def test_full_size_against_reference_digests(ctx, dtab):
    d = digests()["flexicubes_full64"]
    coords, raw = workloads.flexicubes_input(d["parent_res"], d["seed"])
    got = run(ctx, dtab, coords, raw)
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).astype("<i4").tobytes()).hexdigest()
    for k in ("surface", "cases", "edges"):
        assert sha(got[k]) == d[k], k
    assert len(got["vertices"]) == d["n_vertices"] and len(got["faces"]) == d["n_faces"]
    exp = oracle.flexicubes(raw, coords, tables())
    assert sha(exp["faces"]) == d["faces"]
    compare(got, exp, coords, raw, tables())


def test_deterministic(ctx, dtab):
    coords, raw = cases()["noisy16"]
    a, b = run(ctx, dtab, coords, raw), run(ctx, dtab, coords, raw)
    for k in a:
        assert np.array_equal(a[k], b[k]), k


@pytest.mark.parametrize("bad,msg", [
    (np.array([[0, 1, 2, 3], [1, 0, 0, 0]], np.int32), "batch one"),
    (np.array([[0, 1, 2, 3], [0, 0, 256, 0]], np.int32), "outside resolution 256"),
    (np.array([[0, 1, 2, 3], [0, 0, -1, 0]], np.int32), "outside resolution 256"),
    (np.array([[0, 1, 2, 3], [0, 4, 4, 4], [0, 1, 2, 3]], np.int32), "duplicate"),
    (np.array([[0, 1, 2, 3], [0, 1, 2, 3], [2, 0, 0, 0]], np.int32), "duplicate"),
    (np.array([[0, 1, 2, 3], [0, 300, 0, 0], [0, 1, 2, 3]], np.int32), "outside resolution 256"),
])
def test_input_errors(ctx, dtab, bad, msg):
    raw = torch.zeros((len(bad), 101), device="cuda")
    with pytest.raises(s3dsp.S3dError, match=msg):
        ctx.flexicubes(dtab, raw, torch.from_numpy(bad).cuda())
    # the context stays usable
    coords, r = cases()["single_cube"]
    run(ctx, dtab, coords, r)


def test_bad_tables_rejected(ctx):
    t = tables()
    nd = t["num_dual"].copy()
    nd[3] = 7
    with pytest.raises(s3dsp.S3dError, match="num_dual"):
        ctx.flexicubes_tables(t["dmc"], nd, t["check"])
