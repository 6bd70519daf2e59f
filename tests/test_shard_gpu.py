"""Morton-slab split of one volume, run on one GPU: every rank's shard in
turn, its halo filled from the other shards' outputs (what the all-to-all
does across GPUs), through shard hashes, s3dsp_kmap_build_subm3_rows and the
bf16 conv. The result equals the whole-volume conv: bit-exactly with 128-row
tiles (a row's offsets are summed in the same order whatever the shard)."""
import numpy as np
import pytest
import torch

import s3dsp
import shard
import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def layers(ctx, c, nl):
    P = s3dsp.PREC_BF16
    ws, bs = [], []
    for i in range(nl):
        w = torch.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(workloads.conv_weight_slat(c, c, 30 + i)), s3dsp.LAYOUT_SLAT_ROW, 27, c,
                         c, P, w)
        ws.append(w)
        bs.append(dev(workloads.normal((c,), 40 + i, 0.1)))
    return ws, bs


def run_global(ctx, coords, x, ws, bs, flags):
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    cur = x
    for w, b in zip(ws, bs):
        out = torch.empty_like(cur)
        ctx.conv(k, 27, s3dsp.PREC_BF16, cur, w, b, out, cur.shape[1], flags=flags | s3dsp.EPI_SILU)
        cur = out
    return cur.float().cpu().numpy()


def run_sharded(ctx, coords, x, ws, bs, world, flags):
    plans = shard.plan_halos(coords, world)
    c = x.shape[1]
    kms, hs = [], []
    for p in plans:
        h = ctx.hash_build(dev(p.shard_coords(coords)))
        kms.append(ctx.kmap_subm3_rows(h, p.n_own))
        hs.append(h)
    glob = x.clone()  # current layer input, global row order
    for w, b in zip(ws, bs):
        nxt = torch.empty_like(glob)
        for p, k in zip(plans, kms):
            rows = torch.as_tensor(np.concatenate([p.own, p.ghost]), device="cuda")
            xs = glob.index_select(0, rows)  # own rows, then the halo
            out = torch.empty((p.n_own, c), dtype=x.dtype, device="cuda")
            ctx.conv(k, 27, s3dsp.PREC_BF16, xs, w, b, out, c, flags=flags | s3dsp.EPI_SILU)
            nxt[torch.as_tensor(p.own, device="cuda")] = out
        glob = nxt
    return glob.float().cpu().numpy(), plans


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_equals_global_tile128(ctx, world):
    coords = workloads.ellipsoid_shell(40, 2)
    c = 64
    x = dev(workloads.normal((len(coords), c), 3)).to(torch.bfloat16)
    ws, bs = layers(ctx, c, 3)
    ref = run_global(ctx, coords, x, ws, bs, s3dsp.CONV_TILE128)
    got, plans = run_sharded(ctx, coords, x, ws, bs, world, s3dsp.CONV_TILE128)
    assert sum(p.n_own for p in plans) == len(coords)
    assert np.array_equal(got, ref)


def test_sharded_default_dispatch(ctx):
    coords = workloads.ellipsoid_shell(96, 5)  # large enough for the stream-K kernel on the whole volume
    c = 128
    x = dev(workloads.normal((len(coords), c), 6)).to(torch.bfloat16)
    ws, bs = layers(ctx, c, 2)
    ref = run_global(ctx, coords, x, ws, bs, 0)
    got, _ = run_sharded(ctx, coords, x, ws, bs, 4, 0)
    # different kernels / split-tile sums on the two sides: bf16 output rounding
    rel = np.sqrt(((got.astype(np.float64) - ref) ** 2).sum() / (ref.astype(np.float64) ** 2).sum())
    assert rel < 1e-2


@pytest.mark.parametrize("world", [2, 4])
def test_interior_then_boundary_maps(ctx, world):
    """A shard's own rows as two maps (interior rows, which need no halo, and
    boundary rows) over the same [own | ghost] input: what a rank computes
    while its halo is in flight, then after it lands."""
    coords = workloads.ellipsoid_shell(40, 3)
    c = 64
    x = dev(workloads.normal((len(coords), c), 4)).to(torch.bfloat16)
    ws, bs = layers(ctx, c, 2)
    ref = run_global(ctx, coords, x, ws, bs, s3dsp.CONV_TILE128)
    plans = shard.plan_halos(coords, world)
    glob = x.clone()
    maps = []
    for p in plans:
        h = ctx.hash_build(dev(p.shard_coords(coords)))
        ki = ctx.kmap_subm3_range(h, 0, p.n_interior) if p.n_interior > 0 else None
        kb = ctx.kmap_subm3_range(h, p.n_interior, p.n_own)
        maps.append((h, ki, kb))
    assert any(p.n_interior > 0 for p in plans)
    for w, b in zip(ws, bs):
        nxt = torch.empty_like(glob)
        for p, (h, ki, kb) in zip(plans, maps):
            rows = torch.as_tensor(np.concatenate([p.own, p.ghost]), device="cuda")
            xs = glob.index_select(0, rows)
            out = torch.empty((p.n_own, c), dtype=x.dtype, device="cuda")
            f = s3dsp.CONV_TILE128 | s3dsp.EPI_SILU
            if ki is not None:
                ctx.conv(ki, 27, s3dsp.PREC_BF16, xs, w, b, out[:p.n_interior], c, flags=f)
            ctx.conv(kb, 27, s3dsp.PREC_BF16, xs, w, b, out[p.n_interior:], c, flags=f)
            nxt[torch.as_tensor(p.own, device="cuda")] = out
        glob = nxt
    assert np.array_equal(glob.float().cpu().numpy(), ref)
