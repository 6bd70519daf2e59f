"""The SLat generator's sparse stages at their real widths (slat_flow_graph.cpp
:278-296 and :463-531) against the oracle's restatement of the same op
chains: every block alone (128 fine; mean-pool + 128 -> 1024 coarse;
2048-concat coarse -> nearest upsample -> 128; 256-concat -> 128) and the whole
sparse pass, in F32 strict and 3xTF32 (rel-L2 <= 1e-5) and BF16 (<= 1e-2).
The concat and upsample are never built on the device; the pieces that avoid
them (two-source conv and LayerNorm, map composition) are also checked bit for
bit against the same ops on the materialised tensors. Measured rel-L2 values
are printed (pytest -s) so drift toward a gate shows before it fails."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import slat
import workloads
from gates import gate

pytestmark = pytest.mark.gpu

PRECS = [("f32_strict", s3dsp.PREC_F32_STRICT, 1e-5), ("f32_3xtf32", s3dsp.PREC_F32_3XTF32, 1e-5),
         ("bf16", s3dsp.PREC_BF16, 1e-2)]


def rel_l2(got, exp):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    return float(np.sqrt(((got - exp) ** 2).sum()) / max(np.sqrt((exp ** 2).sum()), np.finfo(np.float64).tiny))


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


@pytest.fixture(scope="module")
def case():
    coords = workloads.ellipsoid_shell(32, 1)
    params = slat.slat_params(0)
    mods = slat.slat_mods(0)
    x = workloads.normal((len(coords), slat.IN_CH), 3)
    taps = {}
    exp = oracle.slat_sparse_forward(coords, x, params, mods, accum64=True, taps=taps)
    t = oracle.slat_tables(coords)
    return dict(coords=coords, params=params, mods=mods, x=x, exp=exp, taps=taps, tables=t)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name,prec,tol", PRECS)
def test_sparse_pass_end_to_end(ctx, case, name, prec, tol):
    st = slat.SlatSparse(s3dsp, ctx, case["params"], prec, torch.device("cuda", 0))
    tb = slat.SlatTablesDev(s3dsp, ctx, dev(case["coords"]), torch)
    mods = st.mods_to_device(case["mods"])
    out = st.forward(tb, dev(case["x"]), mods)
    torch.cuda.synchronize()
    ctx.check()
    err = rel_l2(out.cpu().numpy(), case["exp"])
    print(f"\nSLat sparse pass {name}: rel-L2 {err:.3e} (gate {tol:g}), nf {tb.nf}, nc {tb.nc}")
    tb.free()
    gate(err, tol * (1 + 1e-12), name)


def _block_inputs(case, name):
    """The block's input(s) from the oracle chain, and its map / upsample rows."""
    t, taps = case["tables"], case["taps"]
    nf = len(case["coords"])
    nc = len(t["coarse_inv_count"])
    fine = t["conv_fine"].reshape(nf, 27)
    coarse = t["conv_coarse"].reshape(nc, 27)
    if name == "input_blocks.0":
        h = oracle.linear(case["x"], case["params"]["input_layer"]["w"], case["params"]["input_layer"]["b"])
        return h, None, fine, None
    if name == "input_blocks.1":
        d = oracle.downsample_mean(taps["skip0"], t["coarse_children"], t["coarse_inv_count"])
        return d, None, coarse, None
    if name == "out_blocks.0":
        return taps["skip1"], taps["skip1"], fine, t["fine_to_coarse"]
    return taps["out_blocks0"], taps["skip0"], fine, None


@pytest.mark.parametrize("block", list(slat.BLOCKS))
@pytest.mark.parametrize("name,prec,tol", PRECS)
def test_block_at_real_width(ctx, case, block, name, prec, tol):
    xa, xb, nbr, up = _block_inputs(case, block)
    b = case["params"][block]
    sc, sh = case["mods"][block]
    xin = xa if xb is None else np.concatenate([xa, xb], axis=1)
    if up is not None:
        xin = oracle.upsample_nearest(xin, up)
    exp = oracle.slat_res_block(xin, nbr, b["norm1_w"], b["norm1_b"], b["conv1_w"], b["conv1_b"], sc, sh,
                                b["conv2_w"], b["conv2_b"], b.get("skip_w"), b.get("skip_b"), accum64=True)
    st = slat.SlatSparse(s3dsp, ctx, case["params"], prec, torch.device("cuda", 0))
    tb = slat.SlatTablesDev(s3dsp, ctx, dev(case["coords"]), torch)
    kmap = tb.coarse if block == "input_blocks.1" else tb.fine
    mods = st.mods_to_device(case["mods"])
    got = st._block(block, kmap, dev(xa), None if xb is None else dev(xb), mods, len(nbr),
                    up_rows=tb.f2c if up is not None else None)
    torch.cuda.synchronize()
    ctx.check()
    err = rel_l2(got.cpu().numpy(), exp)
    ca, cb, co = slat.BLOCKS[block]
    print(f"\n{block} ({ca}{'+' + str(cb) if cb else ''} -> {co}) {name}: rel-L2 {err:.3e} (gate {tol:g})")
    tb.free()
    gate(err, tol * (1 + 1e-12), f"{block} {name}")


@pytest.mark.parametrize("prec,dt", [(s3dsp.PREC_BF16, torch.bfloat16), (s3dsp.PREC_F32_STRICT, torch.float32),
                                     (s3dsp.PREC_F32_3XTF32, torch.float32)])
@pytest.mark.parametrize("ca,cb,cout", [(1024, 1024, 128), (128, 128, 128), (64, 192, 96)])
def test_conv_concat_equals_conv_of_concat(ctx, prec, dt, ca, cb, cout):
    """Bit for bit: the two-source conv is the one-source conv on the built concat."""
    coords = workloads.ellipsoid_shell(32, 2)
    n = len(coords)
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn((n, ca), generator=g, device="cuda").to(dt)
    b = torch.randn((n, cb), generator=g, device="cuda").to(dt)
    w = torch.empty(s3dsp.Context.packed_bytes(prec, 27, ca + cb, cout), dtype=torch.uint8, device="cuda")
    ctx.weights_pack(torch.from_numpy(workloads.conv_weight_slat(ca + cb, cout, 9)), s3dsp.LAYOUT_SLAT_ROW, 27,
                     ca + cb, cout, prec, w)
    bias = dev(workloads.normal((cout,), 4, 0.1))
    o1 = torch.empty((n, cout), device="cuda")
    o2 = torch.empty((n, cout), device="cuda")
    ctx.conv_concat(k, 27, prec, a, b, w, bias, o1, cout)
    ctx.conv(k, 27, prec, torch.cat([a, b], dim=1).contiguous(), w, bias, o2, cout)
    # the identity map (a Linear) too
    wl = torch.empty(s3dsp.Context.packed_bytes(prec, 1, ca + cb, cout), dtype=torch.uint8, device="cuda")
    ctx.weights_pack(torch.from_numpy(workloads.normal((cout, ca + cb), 6, 0.05)), s3dsp.LAYOUT_LINEAR, 1, ca + cb,
                     cout, prec, wl)
    l1 = torch.empty((n, cout), device="cuda")
    l2 = torch.empty((n, cout), device="cuda")
    ctx.conv_concat(None, 1, prec, a, b, wl, bias, l1, cout)
    ctx.conv(None, 1, prec, torch.cat([a, b], dim=1).contiguous(), wl, bias, l2, cout)
    torch.cuda.synchronize()
    ctx.check()
    assert torch.equal(o1, o2)
    assert torch.equal(l1, l2)


def test_layer_norm_concat_equals_layer_norm_of_concat(ctx):
    g = torch.Generator(device="cuda").manual_seed(8)
    a = torch.randn((3001, 1024), generator=g, device="cuda")
    b = torch.randn((3001, 1024), generator=g, device="cuda") * 2 + 0.5
    gamma = torch.randn(2048, generator=g, device="cuda")
    beta = torch.randn(2048, generator=g, device="cuda")
    for yd in (torch.float32, torch.bfloat16):
        y1 = torch.empty((3001, 2048), dtype=yd, device="cuda")
        y2 = torch.empty_like(y1)
        ctx.layer_norm_concat(a, b, 1e-6, y1, gamma, beta, silu=True)
        ctx.layer_norm(torch.cat([a, b], 1).contiguous(), 1e-6, y2, gamma, beta, silu=True)
        torch.cuda.synchronize()
        assert torch.equal(y1, y2)


def test_kmap_compose_reads_through_rows(ctx, case):
    coords = case["coords"]
    t = case["tables"]
    nf = len(coords)
    nc = len(t["coarse_inv_count"])
    tb = slat.SlatTablesDev(s3dsp, ctx, dev(coords), torch)
    kc = ctx.kmap_compose(tb.fine, tb.f2c, nc)
    dense = torch.empty((nf, 27), dtype=torch.int32, device="cuda")
    ctx.kmap_export_dense(kc, s3dsp.SENTINEL_MESH_NEG1, dense)
    torch.cuda.synchronize()
    ctx.check()
    fine = t["conv_fine"].reshape(nf, 27)
    exp = np.where(fine < nf, t["fine_to_coarse"][np.minimum(fine, nf - 1)], -1)
    assert np.array_equal(dense.cpu().numpy(), exp)
    kc.free()
    tb.free()
