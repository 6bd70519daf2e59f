"""Host logic of the Morton-slab split of one volume across ranks (CPU):
Morton order, halo plan against brute force, the halo all-to-all on gloo
ranks, and a sharded two-layer conv (oracle) equal to the global one."""
import os
import sys

import numpy as np
import pytest

import oracle
import shard
import workloads

HERE = os.path.dirname(os.path.abspath(__file__))


def test_morton_interleave():
    c = np.array([[0, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1], [0, 3, 5, 6]], dtype=np.int32)
    code = shard.morton_codes(c).tolist()
    assert code[:4] == [0, 4, 2, 1]
    # x=011, y=101, z=110 -> bits (x y z) per level, high to low: 0 1 1 | 1 0 1 | 1 1 0
    assert code[4] == 0b011101110


def test_assign_objects_lpt():
    sizes = [5, 9, 1, 7, 3, 8, 2, 6]
    parts = shard.assign_objects(sizes, 3)
    assert sorted(i for p in parts for i in p) == list(range(len(sizes)))
    loads = [sum(sizes[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(sizes)
    assert parts == shard.assign_objects(sizes, 3)  # deterministic
    assert shard.assign_objects(sizes, 1) == [sorted(range(8), key=lambda j: -sizes[j])]
    # 64 shells over 8 ranks: within a few percent of perfect balance
    import workloads
    sz = [len(workloads.ellipsoid_shell(32, s)) for s in range(64)]
    loads = [sum(sz[i] for i in p) for p in shard.assign_objects(sz, 8)]
    assert max(loads) / (sum(sz) / 8) < 1.05


def test_slab_bounds():
    assert shard.slab_bounds(10, 3).tolist() == [0, 3, 6, 10]
    b = shard.slab_bounds(1001, 8)
    assert b[0] == 0 and b[-1] == 1001 and np.diff(b).max() - np.diff(b).min() <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 5])
def test_plan_matches_bruteforce(world):
    coords = workloads.ellipsoid_shell(24, 3)
    n = len(coords)
    plans = shard.plan_halos(coords, world)
    own_all = np.concatenate([p.own for p in plans])
    assert sorted(own_all.tolist()) == list(range(n))
    owner = np.empty(n, dtype=np.int64)
    for p in plans:
        owner[p.own] = p.rank
    index = {tuple(c[1:]): i for i, c in enumerate(coords)}
    offs = [(dx, dy, dz) for dx in (-1, 0, 1) for dy in (-1, 0, 1) for dz in (-1, 0, 1) if (dx, dy, dz) != (0, 0, 0)]
    for p in plans:
        want = set()
        for i in p.own:
            x, y, z = coords[i][1:]
            for dx, dy, dz in offs:
                j = index.get((x + dx, y + dy, z + dz))
                if j is not None and owner[j] != p.rank:
                    want.add(j)
        # own rows: interior (no neighbour on another rank) first, then boundary
        for pos_, i in enumerate(p.own):
            x, y, z = coords[i][1:]
            remote = any((j := index.get((x + dx, y + dy, z + dz))) is not None and owner[j] != p.rank
                         for dx, dy, dz in offs)
            assert remote == (pos_ >= p.n_interior)
        assert set(p.ghost.tolist()) == want
        assert len(p.ghost) == len(want)
        assert p.recv_counts.sum() == p.n_ghost
        assert p.recv_counts[p.rank] == 0
        # grouped by owner, owners ascending
        assert np.all(np.diff(owner[p.ghost]) >= 0)
    # rank q's send list to r is rank r's ghost list from q, same order
    for r in plans:
        for q in plans:
            if q.rank == r.rank:
                continue
            lo = int(r.recv_counts[:q.rank].sum())
            ghosts_from_q = r.ghost[lo:lo + r.recv_counts[q.rank]]
            lo_s = int(q.send_counts[:r.rank].sum())
            sent = q.own[q.send_rows[lo_s:lo_s + q.send_counts[r.rank]]]
            assert np.array_equal(ghosts_from_q, sent)


def _worker(rank, world, port, coords, feats, w, b, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = shard.plan_halos(coords, world)[rank]
        sc = plan.shard_coords(coords)
        nbr = oracle.slat_tables(sc)["conv_fine"].reshape(len(sc), 27)
        # the halo all-to-all alone
        x = torch.zeros((plan.n_own + plan.n_ghost, feats.shape[1]), dtype=torch.float32)
        x[:plan.n_own] = torch.from_numpy(feats[plan.own])
        shard.exchange_halo(x, plan)
        ok_halo = bool(np.array_equal(x[plan.n_own:].numpy(), feats[plan.ghost]))
        # two conv layers, halo refreshed before each
        cur = feats[plan.own]
        for layer in range(2):
            x = torch.zeros((plan.n_own + plan.n_ghost, feats.shape[1]), dtype=torch.float32)
            x[:plan.n_own] = torch.from_numpy(cur)
            shard.exchange_halo(x, plan)
            y = oracle.subm_conv_slat(x.numpy(), nbr, w[layer], b[layer])
            cur = np.ascontiguousarray(y[:plan.n_own])
        result_q.put((rank, ok_halo, plan.own, cur))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_conv_equals_global(world):
    import socket
    import torch.multiprocessing as mp
    coords = workloads.ellipsoid_shell(20, 4)
    n, c = len(coords), 16
    feats = workloads.normal((n, c), 5)
    w = [workloads.conv_weight_slat(c, c, 6 + i) for i in range(2)]
    b = [workloads.normal((c,), 8 + i, 0.1) for i in range(2)]
    nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
    ref = feats
    for layer in range(2):
        ref = oracle.subm_conv_slat(ref, nbr, w[layer], b[layer])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, coords, feats, w, b, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = np.zeros_like(ref)
    for _ in range(world):
        rank, ok_halo, own, out = q.get(timeout=120)
        assert ok_halo, f"rank {rank}: ghost rows differ from the owners' rows"
        got[own] = out
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got, ref)
