"""A compiled C++ host of the C ABI (tests/capi_decode_level.cpp, built by
tests/Makefile; it includes only include/s3dsp.h and links only libs3dsp.so)
runs one mesh upsample level and one config-2 residual block from host
buffers, step by step -- hash, subdivide / kernel map, GroupNorm, convs -- the
way sam3d.cpp's decode_object_mesh would (session.cpp:927-962), and writes
SAMT files. Its outputs must equal, bit for bit, the same work done through
the ctypes binding (the library's block drivers), and match the oracle within
the BF16 gate."""
import os
import subprocess

import numpy as np
import pytest
import torch

import oracle
import s3dsp
import stack
import workloads
from gates import gate

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))


def test_cpp_host_matches_ctypes(tmp_path):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests"), "capi_decode_level"], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    d = str(tmp_path)
    # one mesh upsample level: 128 -> 64 on a 32^3 shell's parents (all 8 children kept)
    parents = workloads.ellipsoid_shell(32, 4)
    cin, cout = 128, 64
    lp = stack._level(cin, cout, 11)
    x = workloads.normal((len(parents), cin), 12)
    for name, a in [("parents", parents), ("x", x)] + list(lp.items()):
        s3dsp.samt_write(os.path.join(d, f"level_{name}.samt"), np.ascontiguousarray(a.reshape(cout, cin))
                         if name == "skip_w" else a)
    # one config-2 block at C = 128 on a 48^3 shell
    cfg = workloads.config2(seed=5, channels=128)
    cfg["coords"] = workloads.ellipsoid_shell(48, 5)
    n, c = len(cfg["coords"]), 128
    cfg["feats"] = workloads.normal((n, c), 6)
    for name in ("coords", "w1", "b1", "gamma", "beta", "w2", "b2"):
        s3dsp.samt_write(os.path.join(d, f"block_{name}.samt"), cfg[name])
    s3dsp.samt_write(os.path.join(d, "block_x.samt"), cfg["feats"])

    r = subprocess.run([os.path.join(ROOT, "tests", "capi_decode_level"), d], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    got_child, _ = s3dsp.samt_read(os.path.join(d, "out_level_child_coords.samt"))
    got_level, _ = s3dsp.samt_read(os.path.join(d, "out_level.samt"))
    got_block, _ = s3dsp.samt_read(os.path.join(d, "out_block.samt"))

    # the same work through the ctypes binding
    ctx = s3dsp.Context(0)
    P = s3dsp.PREC_BF16
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731

    def pack(w, layout, kvol, ci, co):
        dst = torch.empty(s3dsp.Context.packed_bytes(P, kvol, ci, co), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(np.ascontiguousarray(w)), layout, kvol, ci, co, P, dst)
        return dst

    h = ctx.hash_build(dev(parents), reject_duplicates=True)
    nc = 8 * len(parents)
    child = torch.empty((nc, 4), dtype=torch.int32, device="cuda")
    out_level = torch.empty((nc, cout), device="cuda")
    ctx.mesh_upsample_level(h, P, dev(x), cout, dev(lp["gn1_w"]), dev(lp["gn1_b"]),
                            pack(lp["conv1_w"], s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout), dev(lp["conv1_b"]),
                            dev(lp["gn2_w"]), dev(lp["gn2_b"]),
                            pack(lp["conv2_w"], s3dsp.LAYOUT_MESH_PACKED, 27, cout, cout), dev(lp["conv2_b"]),
                            pack(lp["skip_w"].reshape(cout, cin), s3dsp.LAYOUT_LINEAR, 1, cin, cout),
                            dev(lp["skip_b"]), child, out_level)
    hb = ctx.hash_build(dev(cfg["coords"]))
    k = ctx.kmap_subm3(hb)
    out_block = torch.empty((n, c), device="cuda")
    ctx.res_block_gn(k, P, dev(cfg["feats"]), pack(cfg["w1"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c), dev(cfg["b1"]),
                     dev(cfg["gamma"]), dev(cfg["beta"]), pack(cfg["w2"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c),
                     dev(cfg["b2"]), out_block)
    torch.cuda.synchronize()
    ctx.check()
    assert np.array_equal(got_child, child.cpu().numpy())
    assert np.array_equal(got_level, out_level.cpu().numpy())
    assert np.array_equal(got_block, out_block.cpu().numpy())

    # and the oracle, within the BF16 gate
    cc, nb = oracle.mesh_subdivide(parents)
    assert np.array_equal(got_child, cc)
    exp_level = oracle.mesh_upsample_level(x, nb, dict(lp, skip_w=lp["skip_w"].reshape(1, cout * cin)))
    nbr = oracle.slat_tables(cfg["coords"])["conv_fine"].reshape(n, 27)
    exp_block = oracle.resblock_gn(cfg["feats"], nbr, cfg["w1"], cfg["b1"], cfg["gamma"], cfg["beta"], cfg["w2"],
                                   cfg["b2"])
    e1, e2 = rel_l2(got_level, exp_level), rel_l2(got_block, exp_block)
    print(f"\nC++ host: level rel-L2 {e1:.3e}, block rel-L2 {e2:.3e} (BF16 gate 1e-2)")
    gate(e1, 1e-2, "C++ host, level")
    gate(e2, 1e-2, "C++ host, block")
