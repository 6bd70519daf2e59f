"""s3dsp_shard_plan_morton (the C-ABI Morton-slab plan) is identical to
shard.plan_halos: own rows (interior first), ghosts, recv / send counts and
send rows, for several worlds and coordinate sets. Host only, no GPU."""
import numpy as np
import pytest

import s3dsp
import shard
import workloads


def cases():
    shell = workloads.ellipsoid_shell(48, 2)
    rng = np.random.default_rng(3)
    shuffled = shell[rng.permutation(len(shell))]
    neg = np.array([[0, x, y, z] for x in range(-6, 5) for y in range(-4, 7) for z in range(-9, 2)
                    if (x * x + y * y + z * z) % 3], np.int32)
    return {"shell": shell, "shuffled": np.ascontiguousarray(shuffled), "negative": neg}


@pytest.mark.parametrize("name", list(cases()))
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_plan_matches_python(name, world):
    coords = cases()[name]
    for r, p in enumerate(shard.plan_halos(coords, world)):
        c = s3dsp.ShardPlan(coords, world, r)
        assert c.n_interior == p.n_interior
        for k in ("own", "ghost", "recv_counts", "send_counts", "send_rows"):
            assert np.array_equal(getattr(c, k), np.asarray(getattr(p, k), np.int64)), (name, world, r, k)
        c.free()


def test_rejects_bad_arguments():
    coords = workloads.ellipsoid_shell(16, 0)
    with pytest.raises(s3dsp.S3dError):
        s3dsp.ShardPlan(coords, 2, 2)
    bad = coords.copy()
    bad[0, 0] = 3
    with pytest.raises(s3dsp.S3dError, match="one object"):
        s3dsp.ShardPlan(bad, 2, 0)
