"""BF16 conv: CTA-pair (tcgen05 cta_group::2) kernel vs the single-CTA kernel
and vs the oracle, over shapes that stress the pair logic (odd tile counts,
ragged Cout, identity maps, subdivide gathers, every epilogue option), each
launch repeated to catch cross-CTA visibility races (results must be
bit-identical from run to run)."""
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


def run(ctx, k, kvol, x, w, b, cout, n_out, single, reps=3, **kw):
    outs = []
    odt = kw.get("out_dtype", torch.float32)
    for _ in range(reps):
        out = torch.empty((n_out, cout), dtype=odt, device="cuda")
        flags = kw.get("flags", 0) | (s3dsp.CONV_TILE128 if single else s3dsp.CONV_CTA_PAIR)
        part = None
        if kw.get("gn"):
            part = torch.zeros(s3dsp.Context.gn_partials_count(n_out, cout, 32), dtype=torch.float64, device="cuda")
        ctx.conv(k, kvol, s3dsp.PREC_BF16, x, w, b, out, cout, in_shift=kw.get("in_shift", 0),
                 residual=kw.get("residual"), res_shift=kw.get("res_shift", 0), flags=flags, gn_partials=part,
                 gn_groups=32 if kw.get("gn") else 0)
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
        if part is not None:
            outs[-1] = (outs[-1], part.cpu().numpy())
    return outs


@pytest.mark.parametrize("cin,cout,res,seed", [(256, 256, 64, 0), (64, 64, 64, 1), (128, 96, 40, 2),
                                               (192, 192, 32, 3), (96, 101, 24, 4), (64, 16, 20, 5)])
def test_pair_matches_single_and_oracle(ctx, cin, cout, res, seed):
    coords = workloads.ellipsoid_shell(res, seed)
    n = len(coords)
    h = ctx.hash_build(dev(coords))
    k = ctx.kmap_subm3(h)
    x = workloads.normal((n, cin), 10 + seed)
    w = workloads.conv_weight_slat(cin, cout, 20 + seed)
    b = workloads.normal((cout,), 30 + seed, 0.1)
    wp = pack(ctx, w, s3dsp.LAYOUT_SLAT_ROW, 27, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    pair = run(ctx, k, 27, xb, wp, dev(b), cout, n, single=False)
    single = run(ctx, k, 27, xb, wp, dev(b), cout, n, single=True)
    for o in pair[1:]:
        assert np.array_equal(o, pair[0]), "pair kernel not deterministic"
    for o in single[1:]:
        assert np.array_equal(o, single[0])
    gate(rel_l2(pair[0], single[0]), 1e-6)
    nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
    gate(rel_l2(pair[0], oracle.subm_conv_slat(x, nbr, w, b, accum64=True)), 1e-2)


def test_pair_epilogue_options_and_subdivide(ctx):
    parents = workloads.ellipsoid_shell(24, 7)  # 8 * np children: odd/even tiles both exercised
    hp = ctx.hash_build(dev(parents), reject_duplicates=True)
    cc = torch.empty((8 * len(parents), 4), dtype=torch.int32, device="cuda")
    k = ctx.subdivide(hp, cc)
    n_out = 8 * len(parents)
    cin, cout = 192, 96
    x = workloads.normal((len(parents), cin), 40)
    w = workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, 41), cin, cout)
    b = workloads.normal((cout,), 42, 0.1)
    res = dev(workloads.normal((len(parents), cout), 43))
    wp = pack(ctx, w, s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    kw = dict(in_shift=3, residual=res, res_shift=3, flags=s3dsp.EPI_SILU, gn=True)
    pair = run(ctx, k, 27, xb, wp, dev(b), cout, n_out, single=False, **dict(kw))
    single = run(ctx, k, 27, xb, wp, dev(b), cout, n_out, single=True, **dict(kw))
    for o in pair[1:]:
        assert np.array_equal(o[0], pair[0][0]) and np.array_equal(o[1], pair[0][1])
    gate(rel_l2(pair[0][0], single[0][0]), 1e-6)
    gate(rel_l2(pair[0][1], single[0][1]), 1e-6)
    _, nb = oracle.mesh_subdivide(parents)
    pre = oracle.subm_conv_mesh(x, nb, w, b, cout, 27, 3, accum64=True) + np.repeat(res.cpu().numpy(), 8, axis=0)
    gate(rel_l2(pair[0][0], oracle.silu(pre)), 1e-2)


def test_pair_identity_linear_bf16_out(ctx):
    n, cin, cout = 3 * 128 + 17, 256, 128  # 4 row tiles -> 2 pairs; ragged last tile
    x = workloads.normal((n, cin), 50)
    w = workloads.normal((cout, cin), 51, 0.05)
    b = workloads.normal((cout,), 52, 0.1)
    wp = pack(ctx, w, s3dsp.LAYOUT_LINEAR, 1, cin, cout)
    xb = dev(x).to(torch.bfloat16)
    pair = run(ctx, None, 1, xb, wp, dev(b), cout, n, single=False, out_dtype=torch.bfloat16)
    single = run(ctx, None, 1, xb, wp, dev(b), cout, n, single=True, out_dtype=torch.bfloat16)
    assert np.array_equal(pair[0], single[0])
    gate(rel_l2(pair[0], oracle.linear(x, w, b)), 1e-2)
