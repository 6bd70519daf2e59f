"""SLat coarse tables, down/up-sample and the block drivers on the GPU,
against the CPU oracle (tables: bit-exact; floats: F32 rel-L2 1e-5, BF16 1e-2)."""
import os

import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from gates import gate

pytestmark = pytest.mark.gpu

F32_TOL, BF16_TOL = 1e-5, 1e-2
PRECS = [(s3dsp.PREC_F32_STRICT, F32_TOL), (s3dsp.PREC_F32_3XTF32, F32_TOL), (s3dsp.PREC_BF16, BF16_TOL)]


def rel_l2(a, e):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    return float(np.sqrt(((a - e) ** 2).sum() / max((e ** 2).sum(), np.finfo(float).tiny)))


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def pack(ctx, w, layout, kvol, cin, cout, prec):
    dst = torch.empty(s3dsp.Context.packed_bytes(prec, kvol, cin, cout), dtype=torch.uint8, device="cuda")
    ctx.weights_pack(torch.from_numpy(np.ascontiguousarray(w)), layout, kvol, cin, cout, prec, dst)
    return dst


def gpu_tables(ctx, coords):
    h = ctx.hash_build(dev(coords))
    t = ctx.slat_tables(h)
    nf, nc = len(coords), t.nc
    f2c = torch.empty(nf, dtype=torch.int32, device="cuda")
    ch = torch.empty(8 * nc, dtype=torch.int32, device="cuda")
    inv = torch.empty(nc, dtype=torch.float32, device="cuda")
    cc = torch.empty((nc, 4), dtype=torch.int32, device="cuda")
    ctx.slat_tables_export(t, f2c, ch, inv, cc)
    conv_c = torch.empty((nc, 27), dtype=torch.int32, device="cuda")
    ctx.kmap_export_dense(t.coarse_kmap, s3dsp.SENTINEL_SLAT_N, conv_c)
    torch.cuda.synchronize()
    return h, t, dict(nc=nc, fine_to_coarse=f2c.cpu().numpy(), coarse_children=ch.cpu().numpy(),
                      coarse_inv_count=inv.cpu().numpy(), coarse_coords=cc.cpu().numpy(),
                      conv_coarse=conv_c.cpu().numpy().reshape(-1))


@pytest.mark.parametrize("seed,res", [(0, 64), (3, 16), (5, 48)])
def test_slat_coarse_tables_bit_exact(ctx, seed, res):
    coords = workloads.ellipsoid_shell(res, seed)
    _, _, got = gpu_tables(ctx, coords)
    exp = oracle.slat_tables(coords)
    assert got["nc"] == exp["nc"]
    for k in ("fine_to_coarse", "coarse_children", "coarse_inv_count", "conv_coarse", "coarse_coords"):
        assert np.array_equal(got[k], exp[k]), k


def test_slat_coarse_tables_edge_cases(ctx, golden_dir):
    g = np.load(os.path.join(golden_dir, "edge_cases.npz"))
    for name in ("multi", "multi_unique", "dup_rows"):
        _, _, got = gpu_tables(ctx, g[name + "_coords"])
        assert got["nc"] == int(g[name + "_nc"]), name
        for k in ("fine_to_coarse", "coarse_children", "coarse_inv_count", "conv_coarse"):
            assert np.array_equal(got[k], g[f"{name}_{k}"]), (name, k)


def test_slat_down_up_sample(ctx):
    coords = workloads.ellipsoid_shell(64, 1)
    h, t, tab = gpu_tables(ctx, coords)
    x = workloads.normal((len(coords), 128), 2)
    y = torch.empty((t.nc, 128), device="cuda")
    ctx.slat_downsample(t, dev(x), y)
    z = torch.empty((len(coords), 128), device="cuda")
    ctx.slat_upsample(t, y, z)
    torch.cuda.synchronize()
    exp_down = oracle.downsample_mean(x, tab["coarse_children"], tab["coarse_inv_count"])
    assert np.array_equal(y.cpu().numpy(), exp_down)  # same op order in f32
    assert np.array_equal(z.cpu().numpy(), oracle.upsample_nearest(exp_down, tab["fine_to_coarse"]))


@pytest.mark.parametrize("prec,tol", PRECS)
def test_res_block_gn_driver(ctx, prec, tol):
    cfg = workloads.config2()
    coords = cfg["coords"]
    n, c = len(coords), cfg["channels"]
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    w1 = pack(ctx, cfg["w1"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c, prec)
    w2 = pack(ctx, cfg["w2"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c, prec)
    out = torch.empty((n, c), device="cuda")
    ctx.res_block_gn(k, prec, dev(cfg["feats"]), w1, dev(cfg["b1"]), dev(cfg["gamma"]), dev(cfg["beta"]), w2,
                     dev(cfg["b2"]), out)
    torch.cuda.synchronize()
    nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
    exp = oracle.resblock_gn(cfg["feats"], nbr, cfg["w1"], cfg["b1"], cfg["gamma"], cfg["beta"], cfg["w2"], cfg["b2"])
    gate(rel_l2(out.cpu().numpy(), exp), tol)
    # host-buffer form: same result
    out_h = torch.empty((n, c), dtype=torch.float32).pin_memory()
    ctx.res_block_gn_host(prec, torch.from_numpy(coords).pin_memory(), torch.from_numpy(cfg["feats"]).pin_memory(), w1,
                          dev(cfg["b1"]), dev(cfg["gamma"]), dev(cfg["beta"]), w2, dev(cfg["b2"]), out_h)
    assert np.array_equal(out_h.numpy(), out.cpu().numpy())


def mesh_params(cin, cout, seed):
    p = dict(gn1_w=workloads.normal((cin,), seed, 0.2) + 1, gn1_b=workloads.normal((cin,), seed + 1, 0.1),
             conv1_w=workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, seed + 2), cin, cout),
             conv1_b=workloads.normal((cout,), seed + 3, 0.1),
             gn2_w=workloads.normal((cout,), seed + 4, 0.2) + 1, gn2_b=workloads.normal((cout,), seed + 5, 0.1),
             conv2_w=workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cout, cout, seed + 6), cout, cout),
             conv2_b=workloads.normal((cout,), seed + 7, 0.1),
             skip_w=workloads.normal((1, cout * cin), seed + 8, float(np.sqrt(1.0 / cin))),
             skip_b=workloads.normal((cout,), seed + 9, 0.1))
    return p


@pytest.mark.parametrize("prec,tol", PRECS)
@pytest.mark.parametrize("cin,cout,res", [(768, 192, 24), (192, 96, 32)])
def test_mesh_upsample_level_driver(ctx, prec, tol, cin, cout, res):
    parents = workloads.ellipsoid_shell(res, 4)
    np_ = len(parents)
    x = workloads.normal((np_, cin), 11)
    p = mesh_params(cin, cout, 20)
    cc_exp, nb = oracle.mesh_subdivide(parents)
    exp = oracle.mesh_upsample_level(x, nb, p)
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    w1 = pack(ctx, p["conv1_w"], s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout, prec)
    w2 = pack(ctx, p["conv2_w"], s3dsp.LAYOUT_MESH_PACKED, 27, cout, cout, prec)
    ws = pack(ctx, p["skip_w"].reshape(cout, cin), s3dsp.LAYOUT_LINEAR, 1, cin, cout, prec)
    d = {k: dev(v) for k, v in p.items() if k.endswith("_b") or k.startswith("gn")}
    cc = torch.empty((8 * np_, 4), dtype=torch.int32, device="cuda")
    out = torch.empty((8 * np_, cout), device="cuda")
    ctx.mesh_upsample_level(hp, prec, dev(x), cout, d["gn1_w"], d["gn1_b"], w1, d["conv1_b"], d["gn2_w"], d["gn2_b"],
                            w2, d["conv2_b"], ws, d["skip_b"], cc, out)
    torch.cuda.synchronize()
    assert np.array_equal(cc.cpu().numpy(), cc_exp)
    gate(rel_l2(out.cpu().numpy(), exp), tol)
    cc_h = torch.empty((8 * np_, 4), dtype=torch.int32).pin_memory()
    out_h = torch.empty((8 * np_, cout), dtype=torch.float32).pin_memory()
    ctx.mesh_upsample_level_host(prec, torch.from_numpy(parents).pin_memory(), torch.from_numpy(x).pin_memory(), cout,
                                 d["gn1_w"], d["gn1_b"], w1, d["conv1_b"], d["gn2_w"], d["gn2_b"], w2, d["conv2_b"], ws,
                                 d["skip_b"], cc_h, out_h)
    assert np.array_equal(cc_h.numpy(), cc_exp)
    assert np.array_equal(out_h.numpy(), out.cpu().numpy())


@pytest.mark.parametrize("prec,tol", PRECS)
@pytest.mark.parametrize("cin,cout", [(128, 128), (256, 128)])
def test_slat_res_block_driver(ctx, prec, tol, cin, cout):
    coords = workloads.ellipsoid_shell(48, 6)
    n = len(coords)
    x = workloads.normal((n, cin), 30)
    n1w, n1b = workloads.normal((cin,), 31, 0.2) + 1, workloads.normal((cin,), 32, 0.1)
    w1 = workloads.conv_weight_slat(cin, cout, 33)
    b1 = workloads.normal((cout,), 34, 0.1)
    ms, msh = workloads.normal((cout,), 35, 0.2), workloads.normal((cout,), 36, 0.2)
    w2 = workloads.conv_weight_slat(cout, cout, 37)
    b2 = workloads.normal((cout,), 38, 0.1)
    sw = workloads.normal((cout, cin), 39, float(np.sqrt(1.0 / cin))) if cin != cout else None
    sb = workloads.normal((cout,), 40, 0.1) if cin != cout else None
    nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
    exp = oracle.slat_res_block(x, nbr, n1w, n1b, w1, b1, ms, msh, w2, b2, sw, sb)
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    out = torch.empty((n, cout), device="cuda")
    ctx.slat_res_block(k, prec, dev(x), cout, dev(n1w), dev(n1b), pack(ctx, w1, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout, prec),
                       dev(b1), dev(ms), dev(msh), pack(ctx, w2, s3dsp.LAYOUT_SLAT_ROW, 27, cout, cout, prec), dev(b2),
                       pack(ctx, sw, s3dsp.LAYOUT_LINEAR, 1, cin, cout, prec) if sw is not None else None,
                       dev(sb) if sb is not None else None, out)
    torch.cuda.synchronize()
    gate(rel_l2(out.cpu().numpy(), exp), tol)


def test_slat_coarse_res_block_through_down_up(ctx):
    """input_blocks.1 shape: downsample fine (128) to the coarse set, then a
    res block 128 -> 256 on the coarse kernel map, then upsample back."""
    coords = workloads.ellipsoid_shell(64, 2)
    h, t, tab = gpu_tables(ctx, coords)
    nf, nc = len(coords), t.nc
    cin, cout = 128, 256
    x = workloads.normal((nf, cin), 50)
    xd = torch.empty((nc, cin), device="cuda")
    ctx.slat_downsample(t, dev(x), xd)
    p = dict(n1w=workloads.normal((cin,), 51, 0.2) + 1, n1b=workloads.normal((cin,), 52, 0.1),
             w1=workloads.conv_weight_slat(cin, cout, 53), b1=workloads.normal((cout,), 54, 0.1),
             ms=workloads.normal((cout,), 55, 0.2), msh=workloads.normal((cout,), 56, 0.2),
             w2=workloads.conv_weight_slat(cout, cout, 57), b2=workloads.normal((cout,), 58, 0.1),
             sw=workloads.normal((cout, cin), 59, float(np.sqrt(1.0 / cin))), sb=workloads.normal((cout,), 60, 0.1))
    prec = s3dsp.PREC_F32_STRICT
    out = torch.empty((nc, cout), device="cuda")
    ctx.slat_res_block(t.coarse_kmap, prec, xd, cout, dev(p["n1w"]), dev(p["n1b"]),
                       pack(ctx, p["w1"], s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout, prec), dev(p["b1"]), dev(p["ms"]),
                       dev(p["msh"]), pack(ctx, p["w2"], s3dsp.LAYOUT_SLAT_ROW, 27, cout, cout, prec), dev(p["b2"]),
                       pack(ctx, p["sw"], s3dsp.LAYOUT_LINEAR, 1, cin, cout, prec), dev(p["sb"]), out)
    up = torch.empty((nf, cout), device="cuda")
    ctx.slat_upsample(t, out, up)
    torch.cuda.synchronize()
    ex_d = oracle.downsample_mean(x, tab["coarse_children"], tab["coarse_inv_count"])
    ex = oracle.slat_res_block(ex_d, tab["conv_coarse"].reshape(nc, 27), p["n1w"], p["n1b"], p["w1"], p["b1"], p["ms"],
                               p["msh"], p["w2"], p["b2"], p["sw"], p["sb"])
    gate(rel_l2(up.cpu().numpy(), oracle.upsample_nearest(ex, tab["fine_to_coarse"])), F32_TOL)
