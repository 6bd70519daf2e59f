"""Config 4 (mesh-decoder-shaped stack: Linear, 4 GN residual blocks at 256,
subdivide to 128 + 2 blocks, subdivide to 64 + 2 blocks, Linear) through the
C-ABI, end to end against the oracle chain: F32-strict within rel-L2 1e-5,
BF16 within rel-L2 1e-2 (the end-to-end parity gates)."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import stack
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


@pytest.fixture(scope="module")
def case():
    coords = workloads.ellipsoid_shell(16, 1)[:300]  # a patch of a shell: 300 -> 2400 -> 19200 rows
    latent = workloads.normal((len(coords), stack.LATENT), 2)
    p = stack.config4_params(0)
    x = oracle.linear(latent, p["lin_in"]["w"], p["lin_in"]["b"])
    cur = coords
    for lv in range(len(stack.WIDTHS)):
        nbr = oracle.slat_tables(cur)["conv_fine"].reshape(len(cur), 27)
        for b in p[f"blocks{lv}"]:
            x = oracle.resblock_gn(x, nbr, b["w1"], b["b1"], b["gamma"], b["beta"], b["w2"], b["b2"])
        if lv + 1 < len(stack.WIDTHS):
            cc, nb = oracle.mesh_subdivide(cur)
            x = oracle.mesh_upsample_level(x, nb, p[f"up{lv + 1}"])
            cur = cc
    ref = oracle.linear(x, p["lin_out"]["w"], p["lin_out"]["b"])
    return coords, latent, p, cur, ref


@pytest.mark.parametrize("prec,tol", [(s3dsp.PREC_F32_STRICT, 1e-5), (s3dsp.PREC_F32_3XTF32, 1e-5), (s3dsp.PREC_BF16, 1e-2)])
def test_config4_end_to_end(ctx, case, prec, tol):
    coords, latent, p, ref_coords, ref = case
    st = stack.Config4Stack(s3dsp, ctx, p, prec, torch.device("cuda"))
    cc, out = st.forward(torch.from_numpy(coords).cuda(), torch.from_numpy(latent).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(cc.cpu().numpy(), ref_coords)
    assert out.shape == (64 * len(coords), stack.HEAD)
    err = rel_l2(out.cpu().numpy(), ref)
    gate(err, tol, "stack end to end")


def test_units():
    n = 1000
    # linear + 8 convs at n, 3 + 4 at 8n, 3 + 4 at 64n, linear at 64n
    assert stack.units(n) == n + 8 * n + 7 * 8 * n + 7 * 64 * n + 64 * n
