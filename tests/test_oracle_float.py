"""The oracle's float ops against independent float64 torch formulations.

GGML (the reference's float backend) cannot be built here, so the float
restatement is parity-unpinned against GGML itself. These tests pin its
SEMANTICS instead: the sparse conv on a coordinate set equals a dense
torch.conv3d over a zero-filled grid evaluated at the active voxels, with the
reference's weight layouts (SLat (Cout,27,Cin) row format and mesh
(27, Cout*Cin) packing) mapped to conv3d's (Cout, Cin, kd, kh, kw); GroupNorm
and LayerNorm equal torch's in float64.
"""
import numpy as np
import pytest
import torch

import oracle
import workloads
from gates import gate


def dense_subm_conv_ref(coords, feats, w_slat, bias, res):
    """float64 dense conv3d of the scattered features, sampled at coords."""
    cout = w_slat.shape[0]
    cin = feats.shape[1]
    grid = torch.zeros((1, cin, res, res, res), dtype=torch.float64)
    c = torch.from_numpy(coords.astype(np.int64))
    grid[0, :, c[:, 1], c[:, 2], c[:, 3]] = torch.from_numpy(feats).double().T
    w = torch.from_numpy(w_slat).double().reshape(cout, 3, 3, 3, cin).permute(0, 4, 1, 2, 3)
    out = torch.nn.functional.conv3d(grid, w, torch.from_numpy(bias).double(), padding=1)
    return out[0, :, c[:, 1], c[:, 2], c[:, 3]].T.numpy()


def rel_l2(a, e):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    return float(np.sqrt(((a - e) ** 2).sum() / max((e ** 2).sum(), np.finfo(float).tiny)))


@pytest.fixture(scope="module")
def small():
    coords = workloads.ellipsoid_shell(24, seed=5)
    t = oracle.slat_tables(coords)
    nbr = t["conv_fine"].reshape(-1, 27)
    return coords, nbr


@pytest.mark.parametrize("cin,cout", [(16, 8), (32, 24)])
def test_slat_conv_equals_dense_conv3d(small, cin, cout):
    coords, nbr = small
    feats = workloads.normal((len(coords), cin), 1)
    w = workloads.conv_weight_slat(cin, cout, 2)
    b = workloads.normal((cout,), 3, 0.1)
    exp = dense_subm_conv_ref(coords, feats, w, b, 24)
    got32 = oracle.subm_conv_slat(feats, nbr, w, b)
    got64 = oracle.subm_conv_slat(feats, nbr, w, b, accum64=True)
    gate(rel_l2(got64, exp), 1e-6)
    gate(rel_l2(got32, exp), 1e-6)


def test_mesh_conv_equals_slat_conv(small):
    """Same weights in the mesh packed layout, per-offset sum order."""
    coords, nbr_slat = small
    n = len(coords)
    nbr_mesh = np.where(nbr_slat >= n, -1, nbr_slat)
    cin, cout = 16, 12
    feats = workloads.normal((n, cin), 4)
    w = workloads.conv_weight_slat(cin, cout, 5)
    b = workloads.normal((cout,), 6, 0.1)
    packed = workloads.slat_to_mesh_packed(w, cin, cout)
    a = oracle.subm_conv_mesh(feats, nbr_mesh, packed, b, cout)
    e = oracle.subm_conv_slat(feats, nbr_slat, w, b, accum64=True)
    gate(rel_l2(a, e), 1e-6)


def test_mesh_subdivided_conv_equals_repeat_then_conv():
    """in_shift 3 (gather the parent row) == conv over repeat_children(x)."""
    parents = workloads.ellipsoid_shell(12, seed=2)
    cc, nb = oracle.mesh_subdivide(parents)
    cin, cout = 8, 8
    x = workloads.normal((len(parents), cin), 7)
    rep = np.repeat(x, 8, axis=0)  # repeat_children: child row p*8+j = parent p
    w = workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, 8), cin, cout)
    b = workloads.normal((cout,), 9, 0.1)
    a = oracle.subm_conv_mesh(x, nb, w, b, cout, 27, gather_shift=3)
    e = oracle.subm_conv_mesh(rep, nb, w, b, cout, 27, gather_shift=0)
    assert np.array_equal(a, e)
    # and the child conv equals a dense conv3d at 2x resolution
    wslat = w.reshape(27, cout, cin).transpose(1, 0, 2).reshape(cout, 27 * cin)
    exp = dense_subm_conv_ref(cc, rep, wslat, b, 24)
    gate(rel_l2(a, exp), 1e-6)


def test_group_norm_equals_torch():
    x = workloads.normal((500, 64), 11) * 3 + 1
    g = workloads.normal((64,), 12)
    b = workloads.normal((64,), 13)
    got = oracle.group_norm(x, 32, 1e-5, g, b, silu=False)
    t = torch.from_numpy(x).double().T.unsqueeze(0)  # (1, C, N)
    exp = torch.nn.functional.group_norm(t, 32, torch.from_numpy(g).double(), torch.from_numpy(b).double(), 1e-5)
    gate(rel_l2(got, exp[0].T.numpy()), 1e-6)
    got_s = oracle.group_norm(x, 32, 1e-5, g, b, silu=True)
    gate(rel_l2(got_s, torch.nn.functional.silu(exp[0].T).numpy()), 1e-6)


def test_layer_norm_modulate_equals_torch():
    x = workloads.normal((300, 48), 14) * 2 - 0.5
    g, b = workloads.normal((48,), 15), workloads.normal((48,), 16)
    s, sh = workloads.normal((48,), 17, 0.2), workloads.normal((48,), 18, 0.2)
    got = oracle.layer_norm(x, 1e-6, g, b, s, sh, silu=True)
    t = torch.nn.functional.layer_norm(torch.from_numpy(x).double(), (48,), torch.from_numpy(g).double(),
                                       torch.from_numpy(b).double(), 1e-6)
    t = t * (1 + torch.from_numpy(s).double()) + torch.from_numpy(sh).double()
    gate(rel_l2(got, torch.nn.functional.silu(t).numpy()), 1e-6)


def test_down_up_sample_semantics():
    coords = workloads.ellipsoid_shell(16, seed=1)
    t = oracle.slat_tables(coords)
    x = workloads.normal((len(coords), 5), 19)
    down = oracle.downsample_mean(x, t["coarse_children"], t["coarse_inv_count"])
    # scatter-mean with the torch quirk: sum / (count + 1)
    f2c = t["fine_to_coarse"]
    sums = np.zeros((t["nc"], 5))
    np.add.at(sums, f2c, x.astype(np.float64))
    cnt = np.bincount(f2c, minlength=t["nc"])
    gate(rel_l2(down, sums / (cnt + 1)[:, None]), 1e-6)
    up = oracle.upsample_nearest(down, f2c)
    assert np.array_equal(up, down[f2c])
