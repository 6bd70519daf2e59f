"""Sparse convolutions and normalisations on the GPU against the CPU oracle.

Parity gates: F32-strict within rel-L2 1e-5, BF16 within
rel-L2 1e-2, both against the oracle's float64-accumulated restatement of the
reference op order. rel-L2 = ||a - e||_2 / max(||e||_2, DBL_MIN) in float64,
max_abs and sign agreement as tests/test_objects_mesh_decoder_parity.cpp:84-110
define them.
"""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from gates import gate

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 1e-2


def rel_l2(a, e):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    return float(np.sqrt(((a - e) ** 2).sum() / max((e ** 2).sum(), np.finfo(float).tiny)))


def sign_agreement(a, e):
    return float(((np.asarray(a) < 0) == (np.asarray(e) < 0)).mean())


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def pack(ctx, w, layout, kvol, cin, cout, prec):
    nbytes = s3dsp.Context.packed_bytes(prec, kvol, cin, cout)
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    ctx.weights_pack(torch.from_numpy(np.ascontiguousarray(w)), layout, kvol, cin, cout, prec, dst)
    return dst


def subm_setup(ctx, coords):
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    t = oracle.slat_tables(coords)
    return h, k, t["conv_fine"].reshape(-1, 27)


@pytest.fixture(scope="module")
def shell(ctx):
    coords = workloads.ellipsoid_shell(64, 0)
    h, k, nbr = subm_setup(ctx, coords)
    return coords, h, k, nbr


def gpu_conv(ctx, k, kvol, prec, x, wpk, bias, cout, n_out, in_shift=0, residual=None, res_shift=0,
             flags=0, out_dtype=torch.float32, gn=None):
    xin = dev(x)
    if prec == s3dsp.PREC_BF16:
        xin = xin.to(torch.bfloat16)
    out = torch.empty((n_out, cout), dtype=out_dtype, device="cuda")
    part = None
    if gn:
        part = torch.zeros(s3dsp.Context.gn_partials_count(n_out, cout, gn), dtype=torch.float64, device="cuda")
    ctx.conv(k, kvol, prec, xin, wpk, dev(bias) if bias is not None else None, out, cout, in_shift=in_shift,
             residual=dev(residual) if residual is not None else None, res_shift=res_shift, flags=flags,
             gn_partials=part, gn_groups=gn or 0)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), part


@pytest.mark.parametrize("prec", [s3dsp.PREC_F32_STRICT, s3dsp.PREC_BF16])
@pytest.mark.parametrize("cin,cout", [(64, 64), (256, 256), (128, 96), (192, 192), (96, 32)])
def test_subm_conv_slat_layout(ctx, shell, prec, cin, cout):
    coords, h, k, nbr = shell
    n = len(coords)
    x = workloads.normal((n, cin), 1)
    w = workloads.conv_weight_slat(cin, cout, 2)
    b = workloads.normal((cout,), 3, 0.1)
    wpk = pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout, prec)
    got, _ = gpu_conv(ctx, k, 27, prec, x, wpk, b, cout, n)
    exp = oracle.subm_conv_slat(x, nbr, w, b, accum64=True)
    err = rel_l2(got, exp)
    assert err < (F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL), err
    assert sign_agreement(got, exp) > 0.99


@pytest.mark.parametrize("prec", [s3dsp.PREC_F32_STRICT, s3dsp.PREC_BF16])
def test_mesh_conv_subdivided_gather(ctx, prec):
    """Level-1-shaped mesh conv: child map of a subdivide, input gathered from
    the parent rows (in_shift 3 == repeat_children), MESH_PACKED weights."""
    parents = workloads.ellipsoid_shell(32, 6)
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(hp, cc)
    _, nb = oracle.mesh_subdivide(parents)
    cin, cout = 192, 96
    x = workloads.normal((len(parents), cin), 4)
    wp = workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, 5), cin, cout)
    b = workloads.normal((cout,), 6, 0.1)
    wpk = pack(ctx, wp, s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout, prec)
    got, _ = gpu_conv(ctx, k, 27, prec, x, wpk, b, cout, len(nb), in_shift=3)
    exp = oracle.subm_conv_mesh(x, nb, wp, b, cout, 27, gather_shift=3, accum64=True)
    gate(rel_l2(got, exp), (F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL))


@pytest.mark.parametrize("prec", [s3dsp.PREC_F32_STRICT, s3dsp.PREC_BF16])
def test_identity_linear_skip_and_head(ctx, prec):
    """kmap NULL: gb_linear (96 -> 101 head) and the mesh 1x1 skip with the
    spconv 1x1 buffer quirk, reading parent rows (in_shift 3)."""
    n, cin, cout = 3000, 96, 101
    x = workloads.normal((n, cin), 7)
    w = workloads.normal((cout, cin), 8, 0.1)
    b = workloads.normal((cout,), 9, 0.1)
    wpk = pack(ctx, w, s3dsp.LAYOUT_LINEAR, 1, cin, cout, prec)
    got, _ = gpu_conv(ctx, None, 1, prec, x, wpk, b, cout, n)
    exp = oracle.linear(x, w, b)
    gate(rel_l2(got, exp), (F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL))
    # 1x1 quirk: the checkpoint buffer (Cout,1,1,1,Cin) is read as (Cin, Cout)
    cin2, cout2 = 192, 96
    raw = workloads.normal((cout2 * cin2,), 10, 0.1)
    eff = raw.reshape(cin2, cout2).T.copy()  # effective (Cout, Cin) matrix
    wpk2 = pack(ctx, raw, s3dsp.LAYOUT_SPCONV_1X1, 1, cin2, cout2, prec)
    xp = workloads.normal((500, cin2), 11)
    got2, _ = gpu_conv(ctx, None, 1, prec, xp, wpk2, None, cout2, 4000, in_shift=3)
    exp2 = oracle.linear(xp, eff, None, row_shift=3)
    gate(rel_l2(got2, exp2), (F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL))


@pytest.mark.parametrize("prec", [s3dsp.PREC_F32_STRICT, s3dsp.PREC_BF16])
def test_transposed_subdivide_conv(ctx, prec):
    """Config 3's learned 2x2x2 transposed conv: child p*8+j = W_j x_p + b,
    i.e. one GEMM onto [Np, 8*Cout] with the child-major output layout."""
    parents = workloads.ellipsoid_shell(32, 1)
    n = len(parents)
    cin, cout = 128, 64
    x = workloads.normal((n, cin), 12)
    w = workloads.normal((8, cout, cin), 13, float(np.sqrt(1.0 / cin)))
    b = workloads.normal((cout,), 14, 0.1)
    wl = w.reshape(8 * cout, cin)
    wpk = pack(ctx, wl, s3dsp.LAYOUT_LINEAR, 1, cin, 8 * cout, prec)
    got, _ = gpu_conv(ctx, None, 1, prec, x, wpk, np.tile(b, 8), 8 * cout, n)
    got = got.reshape(8 * n, cout)
    exp = np.einsum("jdc,pc->pjd", w.astype(np.float64), x.astype(np.float64)).reshape(8 * n, cout) + b
    gate(rel_l2(got, exp), (F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL))


@pytest.mark.parametrize("prec", [s3dsp.PREC_F32_STRICT, s3dsp.PREC_BF16])
def test_conv_epilogue_residual_silu_and_gn_stats(ctx, shell, prec):
    coords, h, k, nbr = shell
    n = len(coords)
    c = 256
    x = workloads.normal((n, c), 15)
    w = workloads.kaiming_normal_slat(c, c, 16)
    b = workloads.normal((c,), 17, 0.1)
    res = workloads.normal((n, c), 18)
    wpk = pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, c, c, prec)
    got, part = gpu_conv(ctx, k, 27, prec, x, wpk, b, c, n, residual=res, gn=32)
    pre = oracle.subm_conv_slat(x, nbr, w, b, accum64=True) + res
    tol = F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL
    gate(rel_l2(got, pre), tol)
    # partial sums -> per-group mean / E[x^2]
    p = part.cpu().numpy().reshape(-1, 32, 2).sum(0)
    grp = pre.reshape(n, 32, c // 32).astype(np.float64)
    gate(rel_l2(p[:, 0], grp.sum((0, 2))), 10 * tol)
    gate(rel_l2(p[:, 1], (grp ** 2).sum((0, 2))), tol)
    got_s, _ = gpu_conv(ctx, k, 27, prec, x, wpk, b, c, n, residual=res, flags=s3dsp.EPI_SILU)
    gate(rel_l2(got_s, oracle.silu(pre)), tol)


def gpu_resblock(ctx, k, cfg, prec):
    """Config 2 block through the C-ABI primitives."""
    n, c = cfg["feats"].shape
    x32 = dev(cfg["feats"])
    w1 = pack(ctx, cfg["w1"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c, prec)
    w2 = pack(ctx, cfg["w2"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c, prec)
    b1, b2 = dev(cfg["b1"]), dev(cfg["b2"])
    gamma, beta = dev(cfg["gamma"]), dev(cfg["beta"])
    part = torch.empty(s3dsp.Context.gn_partials_count(n, c, 32), dtype=torch.float64, device="cuda")
    sub, mul, add = (torch.empty(c, device="cuda") for _ in range(3))
    y1 = torch.empty((n, c), device="cuda")
    out = torch.empty((n, c), device="cuda")
    if prec == s3dsp.PREC_F32_STRICT:
        ctx.conv(k, 27, prec, x32, w1, b1, y1, c, gn_partials=part, gn_groups=32)
        ctx.gn_finalize(part, n, c, 32, 1e-5, gamma, beta, sub, mul, add)
        ctx.conv(k, 27, prec, y1, w2, b2, out, c, residual=x32, flags=s3dsp.PRO_AFFINE_SILU, pro=(sub, mul, add))
    else:
        xb = torch.empty((n, c), dtype=torch.bfloat16, device="cuda")
        ctx.convert(x32, xb)
        ctx.conv(k, 27, prec, xb, w1, b1, y1, c, gn_partials=part, gn_groups=32)
        ctx.gn_finalize(part, n, c, 32, 1e-5, gamma, beta, sub, mul, add)
        hb = torch.empty((n, c), dtype=torch.bfloat16, device="cuda")
        ctx.channel_affine(y1, sub, mul, add, True, hb)
        ctx.conv(k, 27, prec, hb, w2, b2, out, c, residual=x32)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("prec", [s3dsp.PREC_F32_STRICT, s3dsp.PREC_BF16])
def test_config2_resblock(ctx, shell, prec):
    coords, h, k, nbr = shell
    cfg = workloads.config2()
    got = gpu_resblock(ctx, k, cfg, prec)
    exp = oracle.resblock_gn(cfg["feats"], nbr, cfg["w1"], cfg["b1"], cfg["gamma"], cfg["beta"], cfg["w2"],
                             cfg["b2"])
    err = rel_l2(got, exp)
    assert err < (F32_TOL if prec == s3dsp.PREC_F32_STRICT else BF16_TOL), err


def test_layer_norm_modulate_silu(ctx):
    x = workloads.normal((5000, 128), 20) * 2 + 0.3
    g, b = workloads.normal((128,), 21), workloads.normal((128,), 22)
    s, sh = workloads.normal((128,), 23, 0.2), workloads.normal((128,), 24, 0.2)
    y = torch.empty((5000, 128), device="cuda")
    ctx.layer_norm(dev(x), 1e-6, y, dev(g), dev(b), dev(s), dev(sh), silu=True)
    torch.cuda.synchronize()
    exp = oracle.layer_norm(x, 1e-6, g, b, s, sh, silu=True)
    gate(rel_l2(y.cpu().numpy(), exp), F32_TOL)


def test_gn_stats_kernel_matches_oracle(ctx):
    x = workloads.normal((7000, 192), 25) * 1.5 + 0.2
    g, b = workloads.normal((192,), 26), workloads.normal((192,), 27)
    part = torch.empty(s3dsp.Context.gn_partials_count(7000, 192, 32), dtype=torch.float64, device="cuda")
    ctx.gn_stats(dev(x), 32, part)
    sub, mul, add = (torch.empty(192, device="cuda") for _ in range(3))
    ctx.gn_finalize(part, 7000, 192, 32, 1e-5, dev(g), dev(b), sub, mul, add)
    y = torch.empty((7000, 192), device="cuda")
    ctx.channel_affine(dev(x), sub, mul, add, True, y)
    torch.cuda.synchronize()
    exp = oracle.group_norm(x, 32, 1e-5, g, b, silu=True)
    gate(rel_l2(y.cpu().numpy(), exp), F32_TOL)
