"""The GS decoder's Swin torso (gs_decoder_graph.cpp:13-155) through the C ABI
against the oracle's float64 restatement of the same op order: the window
attention alone, two blocks (one of each shift) at every precision (F32 strict
and 3xTF32: rel-L2 <= 1e-5; BF16: <= 1e-2) and all twelve blocks end to end,
plus the bucket-order row gather. Measured rel-L2 values are printed (pytest
-s) so drift toward a gate shows before it fails."""
import numpy as np
import pytest
import torch

import gs
import oracle
import s3dsp
import workloads
from gates import gate

pytestmark = pytest.mark.gpu

PRECS = [("f32_strict", s3dsp.PREC_F32_STRICT, 1e-5), ("f32_3xtf32", s3dsp.PREC_F32_3XTF32, 1e-5),
         ("bf16", s3dsp.PREC_BF16, 1e-2)]


def rel_l2(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    return float(np.sqrt(((got - exp) ** 2).sum() / (exp ** 2).sum()))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def test_gather_rows(ctx):
    g = np.random.default_rng(2)
    x = g.standard_normal((1000, 40)).astype(np.float32)
    rows = g.permutation(1000)[:777].astype(np.int32)
    for dt in (torch.float32, torch.bfloat16):
        y = torch.empty((777, 40), dtype=dt, device="cuda")
        ctx.gather_rows(dev(x), dev(rows), y)
        torch.cuda.synchronize()
        assert torch.equal(y.cpu(), torch.from_numpy(x[rows]).to(dt))
    ctx.check()


@pytest.mark.parametrize("shift", [0, 1])
def test_window_attention(ctx, shift):
    coords = workloads.ellipsoid_shell(32, 1)
    n = len(coords)
    tb = gs.GsTablesDev(s3dsp, ctx, dev(coords), torch)
    bkt, _, buckets = oracle.gs_window_tables(coords, shift)
    assert np.array_equal(tb.bkt[shift].cpu().numpy(), bkt)
    qkv = workloads.normal((n, 3 * gs.C), 9)
    out = torch.empty((n, gs.C), device="cuda")
    ctx.window_attention(dev(qkv), gs.HEADS, tb.windows[shift], out, scatter=tb.bkt[shift])
    torch.cuda.synchronize()
    ctx.check()
    exp = oracle.window_attention(qkv, gs.HEADS, buckets, bkt)
    err = rel_l2(out.cpu().numpy(), exp)
    print(f"\nwindow attention shift {shift}: rel-L2 {err:.3e}, {len(tb.windows[shift])} windows, "
          f"longest {int(buckets[:, 0].max())} tokens")
    gate(err, 1e-5 * (1 + 1e-12))


@pytest.mark.parametrize("name,prec,tol", PRECS)
def test_two_blocks(ctx, name, prec, tol):
    coords = workloads.ellipsoid_shell(32, 1)
    p = gs.gs_params(0, blocks=2)
    x = workloads.normal((len(coords), gs.IN_CH), 3)
    taps = {}
    exp = oracle.gs_torso_forward(coords, x, p, taps=taps)
    tb = gs.GsTablesDev(s3dsp, ctx, dev(coords), torch)
    got_taps = {}
    got = gs.GsTorso(s3dsp, ctx, p, prec, torch.device("cuda", 0)).forward(tb, dev(x), taps=got_taps)
    torch.cuda.synchronize()
    ctx.check()
    for k in ("block0", "block1"):
        e = rel_l2(got_taps[k].cpu().numpy(), taps[k])
        print(f"\nGS torso {name} {k}: rel-L2 {e:.3e} (gate {tol:g})")
        gate(e, tol * (1 + 1e-12))
    err = rel_l2(got.cpu().numpy(), exp)
    print(f"GS torso {name} two blocks + head: rel-L2 {err:.3e} (gate {tol:g})")
    gate(err, tol * (1 + 1e-12))


@pytest.mark.parametrize("name,prec,tol", [PRECS[0], PRECS[2]])
def test_twelve_blocks_end_to_end(ctx, name, prec, tol):
    coords = workloads.ellipsoid_shell(24, 4)
    p = gs.gs_params(1)
    x = workloads.normal((len(coords), gs.IN_CH), 5)
    exp = oracle.gs_torso_forward(coords, x, p)
    tb = gs.GsTablesDev(s3dsp, ctx, dev(coords), torch)
    got = gs.GsTorso(s3dsp, ctx, p, prec, torch.device("cuda", 0)).forward(tb, dev(x))
    torch.cuda.synchronize()
    ctx.check()
    err = rel_l2(got.cpu().numpy(), exp)
    print(f"\nGS torso {name}, 12 blocks, {len(coords)} tokens: rel-L2 {err:.3e} (gate {tol:g})")
    gate(err, tol * (1 + 1e-12))
