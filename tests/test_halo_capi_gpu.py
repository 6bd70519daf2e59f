"""s3dsp_halo_exchange over NCCL between 2 GPUs (one process each): after the
exchange every rank's ghost rows equal the owners' rows, bit for bit, for f32
and bf16 features. Communicators come from s3dsp_nccl_comm_create with an id
shared through the parent process. Skipped with fewer than 2 GPUs."""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _rank(rank, world, uid, q):
    try:
        sys.path.insert(0, os.path.join(os.path.dirname(HERE), "sam3d.cpp_b200"))
        import s3dsp
        import workloads
        torch.cuda.set_device(rank)
        ctx = s3dsp.Context(rank)
        comm = ctx.nccl_comm(world, rank, uid)
        coords = workloads.ellipsoid_shell(96, 1)
        plan = s3dsp.ShardPlan(coords, world, rank)
        ok = True
        for dt in (torch.float32, torch.bfloat16):
            g = torch.from_numpy(workloads.normal((len(coords), 40), 5)).to(dt)
            rows = np.concatenate([plan.own, plan.ghost])
            x = g[torch.from_numpy(plan.own)].cuda()
            x = torch.cat([x, torch.zeros((plan.n_ghost, 40), dtype=dt, device="cuda")])
            ctx.halo_exchange(plan, comm, x)
            torch.cuda.synchronize()
            ok &= bool(torch.equal(x.cpu(), g[torch.from_numpy(rows)]))
        plan.free(ctx)
        s3dsp.load().s3dsp_nccl_comm_free(comm)
        q.put((rank, ok, plan.n_ghost))
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))


def test_halo_exchange_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "sam3d.cpp_b200"))
    import s3dsp
    uid = s3dsp.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
    assert all(isinstance(n, int) and n > 0 for _, _, n in res), res
