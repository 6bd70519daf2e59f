"""BF16 conv, stream-K kernel (256-row tiles split evenly over the
SMs, pieces of a split tile summed in a fixed order) and its split-K pair
form (one cluster of two CTAs per 256-row tile, the kernel offsets split
between them, the two partial sums added in distributed shared memory):
against the 128-row kernel and the oracle, over split and unsplit tiles,
several column blocks, ragged row counts, subdivide gathers and every epilogue
option. Each launch is repeated: results must be bit-identical from run to
run."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from gates import gate

pytestmark = pytest.mark.gpu


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


def pack(ctx, w, layout, kvol, cin, cout):
    P = s3dsp.PREC_BF16
    dst = torch.empty(s3dsp.Context.packed_bytes(P, kvol, cin, cout), dtype=torch.uint8, device="cuda")
    ctx.weights_pack(torch.from_numpy(np.ascontiguousarray(w)), layout, kvol, cin, cout, P, dst)
    return dst


def run(ctx, k, kvol, x, w, b, cout, n_out, flags=s3dsp.CONV_STREAM_K, reps=3, gn=False, out_dtype=torch.float32,
        **kw):
    outs = []
    for _ in range(reps):
        out = torch.empty((n_out, cout), dtype=out_dtype, device="cuda")
        part = None
        if gn:
            part = torch.full((s3dsp.Context.gn_partials_count(n_out, cout, 32),), 7.0, dtype=torch.float64,
                              device="cuda")
        ctx.conv(k, kvol, s3dsp.PREC_BF16, x, w, b, out, cout, flags=kw.get("epi", 0) | flags, gn_partials=part,
                 gn_groups=32 if gn else 0, in_shift=kw.get("in_shift", 0), residual=kw.get("residual"),
                 res_shift=kw.get("res_shift", 0))
        torch.cuda.synchronize()
        o = out.float().cpu().numpy()
        outs.append((o, part.cpu().numpy()) if gn else o)
    return outs


# split tiles sum their pieces in a different order than one TMEM accumulation:
# f32 reordering error ~ sqrt(K) * 2^-24 for K = 27 * cin terms (5e-6 at cin 256)
ORDER_TOL = 2e-5


def same(a, b):
    if isinstance(a, tuple):
        return all(np.array_equal(x, y) for x, y in zip(a, b))
    return np.array_equal(a, b)


# 256- and 128-row work tiles; 256-row tiles on CTA pairs
SK_FLAGS = [s3dsp.CONV_STREAM_K, s3dsp.CONV_STREAM_K128, s3dsp.CONV_SPLIT_PAIRS]


@pytest.mark.parametrize("skflag", SK_FLAGS)
@pytest.mark.parametrize("cin,cout,res,seed", [
    (256, 256, 64, 0),   # config 2 shape: 60 tiles over all SMs, most tiles split
    (64, 64, 64, 1),     # config 1 shape
    (128, 96, 40, 2),
    (192, 320, 24, 3),   # two column blocks (bn 160)
    (96, 101, 16, 4),    # ragged cout, generic write-out
    (64, 16, 8, 5),      # a handful of rows: many pieces per tile
    (256, 512, 20, 6),   # two 256-column blocks
])
def test_sk_matches_tile128_and_oracle(ctx, cin, cout, res, seed, skflag):
    coords = workloads.ellipsoid_shell(res, seed) if res >= 16 else workloads.ellipsoid_shell(16, seed)[:37]
    n = len(coords)
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    x = workloads.normal((n, cin), 10 + seed)
    w = workloads.conv_weight_slat(cin, cout, 20 + seed)
    b = workloads.normal((cout,), 30 + seed, 0.1)
    wp = pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    sk = run(ctx, k, 27, xb, wp, dev(b), cout, n, flags=skflag)
    t128 = run(ctx, k, 27, xb, wp, dev(b), cout, n, flags=s3dsp.CONV_TILE128, reps=1)
    for o in sk[1:]:
        assert np.array_equal(o, sk[0]), "stream-K kernel not deterministic"
    gate(rel_l2(sk[0], t128[0]), ORDER_TOL)
    nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
    gate(rel_l2(sk[0], oracle.subm_conv_slat(x, nbr, w, b, accum64=True)), 1e-2)


@pytest.mark.parametrize("skflag", SK_FLAGS)
@pytest.mark.parametrize("out_dtype,res_dtype,silu", [(torch.float32, torch.float32, True),
                                                      (torch.bfloat16, torch.bfloat16, False),
                                                      (torch.float32, torch.bfloat16, False)])
def test_sk_epilogue_gn_and_subdivide(ctx, out_dtype, res_dtype, silu, skflag):
    parents = workloads.ellipsoid_shell(24, 7)
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(hp, cc)
    n_out = 8 * len(parents)
    cin, cout = 192, 96
    x = workloads.normal((len(parents), cin), 40)
    w = workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, 41), cin, cout)
    b = workloads.normal((cout,), 42, 0.1)
    res = dev(workloads.normal((len(parents), cout), 43)).to(res_dtype)
    wp = pack(ctx, w, s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    kw = dict(in_shift=3, residual=res, res_shift=3, epi=s3dsp.EPI_SILU if silu else 0, gn=True, out_dtype=out_dtype)
    sk = run(ctx, k, 27, xb, wp, dev(b), cout, n_out, flags=skflag, **kw)
    t128 = run(ctx, k, 27, xb, wp, dev(b), cout, n_out, flags=s3dsp.CONV_TILE128, reps=1, **kw)
    for o in sk[1:]:
        assert same(o, sk[0]), "stream-K kernel not deterministic"
    tol = ORDER_TOL if out_dtype == torch.float32 else 1e-2
    gate(rel_l2(sk[0][0], t128[0][0]), tol)
    gate(rel_l2(sk[0][1], t128[0][1]), (ORDER_TOL if out_dtype == torch.float32 else 1e-2))
    _, nb = oracle.mesh_subdivide(parents)
    pre = oracle.subm_conv_mesh(x, nb, w, b, cout, 27, 3, accum64=True) + np.repeat(
        res.float().cpu().numpy(), 8, axis=0)
    # GroupNorm partial sums of the pre-SiLU values, per 128-row tile
    tiles = (n_out + 127) // 128
    exp = np.zeros((tiles, 32, 2))
    for t in range(tiles):
        blk = pre[128 * t:128 * (t + 1)].reshape(-1, 32, cout // 32)
        exp[t, :, 0] = blk.sum(axis=(0, 2))
        exp[t, :, 1] = (blk.astype(np.float64) ** 2).sum(axis=(0, 2))
    gate(rel_l2(sk[0][1].reshape(tiles, 32, 2), exp), 1e-2)
    ref = oracle.silu(pre) if silu else pre
    gate(rel_l2(sk[0][0], ref), 1e-2)


@pytest.mark.parametrize("skflag", [s3dsp.CONV_STREAM_K, s3dsp.CONV_SPLIT_PAIRS])
@pytest.mark.parametrize("n", [1, 255, 256, 257, 3 * 256 + 17, 40000])
def test_sk_identity_linear(ctx, n, skflag):
    cin, cout = 256, 128
    x = workloads.normal((n, cin), 50)
    w = workloads.normal((cout, cin), 51, 0.05)
    b = workloads.normal((cout,), 52, 0.1)
    wp = pack(ctx, w, s3dsp.LAYOUT_LINEAR, 1, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    sk = run(ctx, None, 1, xb, wp, dev(b), cout, n, flags=skflag, out_dtype=torch.bfloat16, reps=2)
    t128 = run(ctx, None, 1, xb, wp, dev(b), cout, n, flags=s3dsp.CONV_TILE128, out_dtype=torch.bfloat16, reps=1)
    assert np.array_equal(sk[0], sk[1])
    if skflag == s3dsp.CONV_STREAM_K:
        assert np.array_equal(sk[0], t128[0])  # whole tiles, same MMA order: bit-identical
    else:
        # CTA pairs split the 4 channel chunks 2 / 2 and add the two halves: f32
        # reordering, then the bf16 rounding of the output
        gate(rel_l2(sk[0], t128[0]), 1e-3)
    gate(rel_l2(sk[0], oracle.linear(x, w, b)), 1e-2)


def test_kernel_choice(ctx):
    P = s3dsp.PREC_BF16
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    pairs = "conv_sk_kernel<256>:pairs"
    assert ctx.conv_kernel(15159, 27, 256, 256, P) == pairs   # config 2: 60 pairs, one wave
    assert ctx.conv_kernel(128 * sms - 5, 27, 256, 256, P) == pairs  # 74 pairs: still one wave
    assert ctx.conv_kernel(34060, 27, 256, 256, P) == pairs   # two waves of pairs
    assert ctx.conv_kernel(3815, 27, 512, 512, P) == "conv_sk_kernel<256>"  # wide: stream-K
    assert ctx.conv_kernel(2153, 27, 1024, 1024, P) == "conv_sk_kernel<256>"
    assert ctx.conv_kernel(128 * sms + 900, 27, 256, 256, P) == "conv_sk_kernel<256>"  # a thin second wave
    assert ctx.conv_kernel(128 * 8 * sms, 27, 256, 256, P) == "conv_sk_kernel<256>"
    assert ctx.conv_kernel(128 * 8 * sms, 1, 256, 256, P) == "conv_tc_kernel"     # linear layers
    assert ctx.conv_kernel(1000, 27, 256, 256, P, s3dsp.CONV_STREAM_K) == "conv_sk_kernel<256>"
    assert ctx.conv_kernel(1000, 27, 256, 256, P, s3dsp.CONV_STREAM_K128) == "conv_sk_kernel<128>"
    assert ctx.conv_kernel(1000, 27, 256, 256, P, s3dsp.CONV_SPLIT_PAIRS) == "conv_sk_kernel<256>:pairs"
    assert ctx.conv_kernel(128 * 3 * sms, 27, 256, 256, P, s3dsp.CONV_TILE128) == "conv_tc_kernel"
    assert ctx.conv_kernel(1000, 27, 256, 256, s3dsp.PREC_F32_STRICT) == "conv_f32_kernel"
