"""BF16 conv, per-tile input halo kernel (each 128-row tile loads its distinct
source rows once into shared memory and builds every offset's A tile from
there): against the 128-row kernel and the oracle, over sorted and shuffled
coordinate lists (tiles whose rows overflow the halo read global memory
instead), one to four 64-channel chunks, ragged widths, subdivide gathers and
every epilogue option. Each launch is repeated: results must be bit-identical
from run to run. With one channel chunk the kernel adds the same products in
the same order as the 128-row kernel, so the outputs are bit-identical to it."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from gates import gate

pytestmark = pytest.mark.gpu

H = s3dsp.CONV_HALO
# more channel chunks: the halo kernel takes the chunks outer and the offsets
# inner (the 128-row kernel the other way round), an f32 reordering of
# 27 * cin products (~sqrt(K) * 2^-24)
ORDER_TOL = 2e-5


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


def run(ctx, k, x, w, b, cout, n_out, flags, reps=3, gn=False, out_dtype=torch.float32, **kw):
    outs = []
    for _ in range(reps):
        out = torch.empty((n_out, cout), dtype=out_dtype, device="cuda")
        part = None
        if gn:
            part = torch.full((s3dsp.Context.gn_partials_count(n_out, cout, 32),), 7.0, dtype=torch.float64,
                              device="cuda")
        ctx.conv(k, 27, s3dsp.PREC_BF16, x, w, b, out, cout, flags=kw.get("epi", 0) | flags, gn_partials=part,
                 gn_groups=32 if gn else 0, in_shift=kw.get("in_shift", 0), residual=kw.get("residual"),
                 res_shift=kw.get("res_shift", 0))
        torch.cuda.synchronize()
        o = out.float().cpu().numpy()
        outs.append((o, part.cpu().numpy()) if gn else o)
    return outs


def same(a, b):
    if isinstance(a, tuple):
        return all(np.array_equal(x, y) for x, y in zip(a, b))
    return np.array_equal(a, b)


@pytest.mark.parametrize("cin,cout,res,seed,shuffle", [
    (64, 64, 64, 0, None),     # config 1 shape: ~430 distinct rows per tile, a few tiles overflow the halo
    (64, 64, 64, 0, "all"),    # unordered list: every tile reads global memory
    (64, 64, 40, 1, "half"),   # the second half unordered: both paths in one launch
    (128, 128, 40, 2, None),   # two chunks, one CTA per SM
    (96, 48, 32, 3, None),     # a half-filled second chunk, 48 columns
    (256, 128, 24, 4, None),   # four chunks
    (192, 100, 20, 5, None),   # ragged cout (112 padded columns), generic write-out
    (192, 42, 20, 5, None),    # ragged cout (48 padded columns), two CTAs per SM
    (256, 64, 24, 4, None),    # four chunks, 64 columns
    (64, 16, 8, 6, None),      # a handful of rows (one partial tile)
])
def test_halo_matches_tile128_and_oracle(ctx, cin, cout, res, seed, shuffle):
    coords = workloads.ellipsoid_shell(res, seed) if res >= 16 else workloads.ellipsoid_shell(16, seed)[:37]
    rng = np.random.default_rng(90 + seed)
    if shuffle == "all":
        coords = coords[rng.permutation(len(coords))]
    elif shuffle == "half":
        h = len(coords) // 2
        coords = np.concatenate([coords[:h], coords[h:][rng.permutation(len(coords) - h)]])
    n = len(coords)
    hsh = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(hsh)
    x = workloads.normal((n, cin), 10 + seed)
    w = workloads.conv_weight_slat(cin, cout, 20 + seed)
    b = workloads.normal((cout,), 30 + seed, 0.1)
    wp = pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    assert ctx.conv_kernel(n, 27, cin, cout, s3dsp.PREC_BF16, H) == "conv_halo_kernel"
    hl = run(ctx, k, xb, wp, dev(b), cout, n, H)
    t128 = run(ctx, k, xb, wp, dev(b), cout, n, s3dsp.CONV_TILE128, reps=1)
    for o in hl[1:]:
        assert np.array_equal(o, hl[0]), "halo kernel not deterministic"
    if cin <= 64:
        assert np.array_equal(hl[0], t128[0]), "one chunk: same products, same order as the 128-row kernel"
    else:
        gate(rel_l2(hl[0], t128[0]), ORDER_TOL)
    nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
    gate(rel_l2(hl[0], oracle.subm_conv_slat(x, nbr, w, b, accum64=True)), 1e-2)


@pytest.mark.parametrize("cin", [64, 128, 192])
@pytest.mark.parametrize("out_dtype,res_dtype,silu", [(torch.float32, torch.float32, True),
                                                      (torch.bfloat16, torch.bfloat16, False),
                                                      (torch.float32, torch.bfloat16, False)])
def test_halo_epilogue_gn_and_subdivide(ctx, cin, out_dtype, res_dtype, silu):
    parents = workloads.ellipsoid_shell(24, 7)
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(hp, cc)
    n_out = 8 * len(parents)
    cout = 96
    x = workloads.normal((len(parents), cin), 40)
    w = workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, 41), cin, cout)
    b = workloads.normal((cout,), 42, 0.1)
    res = dev(workloads.normal((len(parents), cout), 43)).to(res_dtype)
    wp = pack(ctx, w, s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    kw = dict(in_shift=3, residual=res, res_shift=3, epi=s3dsp.EPI_SILU if silu else 0, gn=True, out_dtype=out_dtype)
    hl = run(ctx, k, xb, wp, dev(b), cout, n_out, H, **kw)
    t128 = run(ctx, k, xb, wp, dev(b), cout, n_out, s3dsp.CONV_TILE128, reps=1, **kw)
    for o in hl[1:]:
        assert same(o, hl[0]), "halo kernel not deterministic"
    if cin <= 64:
        assert np.array_equal(hl[0][0], t128[0][0])
        # the GroupNorm column sums run over 16 rows per epilogue warp here
        # (8 in the 128-row kernel) before the warp-order total: f64 reordering
        gate(rel_l2(hl[0][1], t128[0][1]), 1e-12)
    else:
        tol = ORDER_TOL if out_dtype == torch.float32 else 1e-2
        gate(rel_l2(hl[0][0], t128[0][0]), tol)
        gate(rel_l2(hl[0][1], t128[0][1]), tol)
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
    gate(rel_l2(hl[0][1].reshape(tiles, 32, 2), exp), 1e-2)
    ref = oracle.silu(pre) if silu else pre
    gate(rel_l2(hl[0][0], ref), 1e-2)


def test_halo_kernel_choice(ctx):
    P = s3dsp.PREC_BF16
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    # automatic: narrow layers (<= 64 output channels, two CTAs per SM) of at least a wave of tiles
    assert ctx.conv_kernel(970176, 27, 64, 64, P) == "conv_halo_kernel"
    assert ctx.conv_kernel(970176, 27, 128, 64, P, in_shift=3) == "conv_halo_kernel"
    assert ctx.conv_kernel(128 * sms, 27, 64, 64, P) == "conv_halo_kernel"
    assert ctx.conv_kernel(128 * sms - 128, 27, 64, 64, P) != "conv_halo_kernel"
    # a same-level 128 -> 64 conv references ~400 rows per tile: too many for two CTAs per SM
    assert ctx.conv_kernel(970176, 27, 128, 64, P) != "conv_halo_kernel"
    assert ctx.conv_kernel(121272, 27, 128, 128, P) != "conv_halo_kernel"
    # forced
    assert ctx.conv_kernel(970176, 27, 64, 64, P, H) == "conv_halo_kernel"
    assert ctx.conv_kernel(121272, 27, 128, 128, P, H) == "conv_halo_kernel"
    assert ctx.conv_kernel(121272, 27, 256, 128, P, H) == "conv_halo_kernel"
    # layers the kernel does not take fall through to the size-based choice
    assert ctx.conv_kernel(15159, 27, 256, 256, P, H) == "conv_sk_kernel<256>:pairs"
    assert ctx.conv_kernel(15159, 27, 320, 64, P, H) != "conv_halo_kernel"
    assert ctx.conv_kernel(15159, 1, 64, 64, P, H) == "conv_tc_kernel"


@pytest.mark.parametrize("cin,in_shift", [(64, 0), (128, 3)])
def test_halo_auto_on_subdivided_level(ctx, cin, in_shift):
    """A subdivided 64^3 shell (~121k rows, ~950 tiles): the automatic choice
    takes the halo kernel for the C = 64 conv and the 128 -> 64 subdivide conv;
    with GroupNorm partials and SiLU, the outputs match the 128-row kernel
    (bit for bit with one channel chunk)."""
    parents = workloads.ellipsoid_shell(64, 12)
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(hp, cc)
    n_out = 8 * len(parents)
    n_in = len(parents) if in_shift else n_out
    cout = 64
    assert ctx.conv_kernel(n_out, 27, cin, cout, s3dsp.PREC_BF16, in_shift=in_shift) == "conv_halo_kernel"
    x = dev(workloads.normal((n_in, cin), 60)).to(torch.bfloat16)
    w = pack(ctx, workloads.conv_weight_slat(cin, cout, 61), s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout)
    b = dev(workloads.normal((cout,), 62, 0.1))
    kw = dict(in_shift=in_shift, gn=True, epi=s3dsp.EPI_SILU)
    auto = run(ctx, k, x, w, b, cout, n_out, 0, reps=2, **kw)
    t128 = run(ctx, k, x, w, b, cout, n_out, s3dsp.CONV_TILE128, reps=1, **kw)
    assert same(auto[0], auto[1]), "halo kernel not deterministic"
    if cin <= 64:
        assert np.array_equal(auto[0][0], t128[0][0])
    else:
        gate(rel_l2(auto[0][0], t128[0][0]), ORDER_TOL)
    gate(rel_l2(auto[0][1], t128[0][1]), ORDER_TOL)
