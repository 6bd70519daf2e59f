"""GS decoder Swin window tables and APE on the device against the oracle
(itself equal to the reference's own GsTables::build): window buckets
bit-exact for both shifts, the embedding within f32 sin/cos rounding."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
from test_oracle_tables import gs_cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


@pytest.mark.parametrize("name", list(gs_cases()))
def test_window_tables_bit_exact(ctx, name):
    coords = gs_cases()[name]
    d = torch.from_numpy(np.ascontiguousarray(coords)).cuda()
    n = len(coords)
    for si in (0, 1):
        bkt = torch.empty(n, dtype=torch.int32, device="cuda")
        bwd = torch.empty(n, dtype=torch.int32, device="cuda")
        buckets = ctx.gs_window_tables(d, 4 * si, bkt, bwd)
        exp = oracle.gs_window_tables(coords, si)
        assert np.array_equal(bkt.cpu().numpy(), exp[0]), (name, si)
        assert np.array_equal(bwd.cpu().numpy(), exp[1]), (name, si)
        assert np.array_equal(buckets, exp[2]), (name, si)


@pytest.mark.parametrize("name", ["shell64", "negative"])
def test_ape(ctx, name):
    coords = gs_cases()[name]
    d = torch.from_numpy(np.ascontiguousarray(coords)).cuda()
    out = torch.empty((len(coords), 768), device="cuda")
    ctx.ape(d, out)
    got = out.cpu().numpy()
    exp = oracle.ape(coords)
    assert np.abs(got - exp).max() < 1e-6
