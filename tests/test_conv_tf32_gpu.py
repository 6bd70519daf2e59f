"""The 3xTF32 tensor-core convolution (S3DSP_PREC_F32_3XTF32: f32 operands
split into a TF32 high part and its remainder, lo*hi + hi*lo + hi*hi
tcgen05 MMAs into an f32 TMEM accumulator) against the oracle's
float64-accumulated restatement, at the F32 gate (rel-L2 <= 1e-5), and
against the FFMA strict path."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from test_conv_gpu import F32_TOL, dev, gpu_conv, pack, rel_l2, sign_agreement, subm_setup
from gates import gate

pytestmark = pytest.mark.gpu
P = s3dsp.PREC_F32_3XTF32


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


@pytest.fixture(scope="module")
def shell(ctx):
    coords = workloads.ellipsoid_shell(64, 0)
    h, k, nbr = subm_setup(ctx, coords)
    return coords, h, k, nbr


@pytest.mark.parametrize("cin,cout", [(64, 64), (256, 256), (128, 96), (96, 32), (36, 200)])
def test_subm_conv(ctx, shell, cin, cout):
    coords, h, k, nbr = shell
    n = len(coords)
    x = workloads.normal((n, cin), 1)
    w = workloads.conv_weight_slat(cin, cout, 2)
    b = workloads.normal((cout,), 3, 0.1)
    got, _ = gpu_conv(ctx, k, 27, P, x, pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout, P), b, cout, n)
    exp = oracle.subm_conv_slat(x, nbr, w, b, accum64=True)
    gate(rel_l2(got, exp), F32_TOL)
    assert sign_agreement(got, exp) > 0.99
    ffma, _ = gpu_conv(ctx, k, 27, s3dsp.PREC_F32_STRICT, x,
                       pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout, s3dsp.PREC_F32_STRICT), b, cout, n)
    gate(rel_l2(got, ffma), 2 * F32_TOL)


def test_mesh_conv_parent_gather(ctx):
    parents = workloads.ellipsoid_shell(32, 6)
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(hp, cc)
    _, nb = oracle.mesh_subdivide(parents)
    cin, cout = 192, 96
    x = workloads.normal((len(parents), cin), 4)
    wp = workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, 5), cin, cout)
    b = workloads.normal((cout,), 6, 0.1)
    got, _ = gpu_conv(ctx, k, 27, P, x, pack(ctx, wp, s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout, P), b, cout,
                      len(nb), in_shift=3)
    exp = oracle.subm_conv_mesh(x, nb, wp, b, cout, 27, gather_shift=3, accum64=True)
    gate(rel_l2(got, exp), F32_TOL)


def test_identity_linear_head(ctx):
    n, cin, cout = 3000, 96, 101
    x = workloads.normal((n, cin), 7)
    w = workloads.normal((cout, cin), 8, 0.1)
    b = workloads.normal((cout,), 9, 0.1)
    got, _ = gpu_conv(ctx, None, 1, P, x, pack(ctx, w, s3dsp.LAYOUT_LINEAR, 1, cin, cout, P), b, cout, n)
    gate(rel_l2(got, oracle.linear(x, w, b)), F32_TOL)


def test_epilogue_residual_silu_and_gn_stats(ctx, shell):
    coords, h, k, nbr = shell
    n, c = len(coords), 256
    x = workloads.normal((n, c), 15)
    w = workloads.kaiming_normal_slat(c, c, 16)
    b = workloads.normal((c,), 17, 0.1)
    res = workloads.normal((n, c), 18)
    wpk = pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P)
    got, part = gpu_conv(ctx, k, 27, P, x, wpk, b, c, n, residual=res, gn=32)
    pre = oracle.subm_conv_slat(x, nbr, w, b, accum64=True) + res
    gate(rel_l2(got, pre), F32_TOL)
    p = part.cpu().numpy().reshape(-1, 32, 2).sum(0)
    grp = pre.reshape(n, 32, c // 32).astype(np.float64)
    gate(rel_l2(p[:, 1], (grp ** 2).sum((0, 2))), F32_TOL)
    got_s, _ = gpu_conv(ctx, k, 27, P, x, wpk, b, c, n, residual=res, flags=s3dsp.EPI_SILU)
    gate(rel_l2(got_s, oracle.silu(pre)), F32_TOL)


def test_rejects_prologue_pairs_and_bf16(ctx, shell):
    coords, h, k, nbr = shell
    n, c = len(coords), 64
    wpk = pack(ctx, workloads.conv_weight_slat(c, c, 2), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P)
    x = dev(workloads.normal((n, c), 1))
    out = torch.empty((n, c), device="cuda")
    with pytest.raises(s3dsp.S3dError, match="f32 input"):
        ctx.conv(k, 27, P, x.to(torch.bfloat16), wpk, None, out, c)
    with pytest.raises(s3dsp.S3dError, match="CTA pairs"):
        ctx.conv(k, 27, P, x, wpk, None, out, c, flags=s3dsp.CONV_CTA_PAIR)
    assert s3dsp.load().s3dsp_conv_kernel(ctx.handle, n, 27, c, c, P, 0) == b"conv_tc_kernel<tf32x3>"
