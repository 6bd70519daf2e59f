"""GGUF weights on the device: dequantisation of every dtype the reference's
converter writes, bit-exact against gguf-py's numpy statement of GGML's block
formats, and a mesh upsample level (MeshUpsampleGraph::build,
mesh_decoder_graph.cpp:42-132) whose weights come from a synthetic
slat_decoder_mesh GGUF in the converter's layout (convert_sam3d_to_gguf.py:
463-502), against the oracle with the dequantised weights."""
import numpy as np
import pytest
import torch

import oracle
import s3dsp
import workloads
from gguf_fixtures import QTYPES, dequantized, stored, write
from gates import gate

pytestmark = pytest.mark.gpu

PRECS = [(s3dsp.PREC_F32_STRICT, 1e-5), (s3dsp.PREC_BF16, 1e-2)]


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return s3dsp.Context(0)


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("dt", list(QTYPES))
def test_dequantize_bit_exact(ctx, tmp_path, dt):
    x = np.random.default_rng(3).normal(0, 0.2, size=(6, 1024)).astype(np.float32)
    arr, raw = stored(x, dt, seed=4)
    p = str(tmp_path / "t.gguf")
    write(p, {"w": (arr, raw)})
    exp = dequantized(arr, raw).reshape(6, 1024)
    g = s3dsp.Gguf(p)
    got = g.load(ctx, "w").cpu().numpy()
    assert got.shape == exp.shape and np.array_equal(got, exp)
    got16 = g.load(ctx, "w", bf16=True).cpu()
    assert torch.equal(got16, torch.from_numpy(exp).to(torch.bfloat16))
    # the device-to-device form on the raw bytes
    src = torch.from_numpy(g.read("w")).cuda()
    out = torch.empty(exp.size, device="cuda")
    s3dsp._call(s3dsp.load().s3dsp_dequantize, ctx.handle, g.info("w")["type"], s3dsp.ptr(src), exp.size, s3dsp.F32,
                s3dsp.ptr(out))
    assert np.array_equal(out.cpu().numpy().reshape(exp.shape), exp)


def mesh_level_gguf(path, cin, cout, dtype, seed, level=1):
    """A slat_decoder_mesh-style GGUF holding one upsample level; returns the
    dequantised parameters in the oracle's layout."""
    rng = np.random.default_rng(seed)
    pre = f"meshdec.upsample.{level}."
    p32 = dict(gn1_w=rng.normal(1, 0.2, cin), gn1_b=rng.normal(0, 0.1, cin),
               conv1_w=workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, seed + 1), cin, cout),
               conv1_b=rng.normal(0, 0.1, cout), gn2_w=rng.normal(1, 0.2, cout), gn2_b=rng.normal(0, 0.1, cout),
               conv2_w=workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cout, cout, seed + 2), cout, cout),
               conv2_b=rng.normal(0, 0.1, cout),
               skip_w=rng.normal(0, float(np.sqrt(1.0 / cin)), (1, cout * cin)), skip_b=rng.normal(0, 0.1, cout))
    names = dict(gn1_w="act_layers.0.weight", gn1_b="act_layers.0.bias", conv1_w="out_layers.0.conv.weight",
                 conv1_b="out_layers.0.conv.bias", gn2_w="out_layers.1.weight", gn2_b="out_layers.1.bias",
                 conv2_w="out_layers.3.conv.weight", conv2_b="out_layers.3.conv.bias",
                 skip_w="skip_connection.conv.weight", skip_b="skip_connection.conv.bias")
    tensors, deq = {}, {}
    for i, (k, v) in enumerate(p32.items()):
        v = np.ascontiguousarray(v, np.float32)
        if v.ndim == 1:  # the converter keeps 1-D parameters in F32 (gguf_schema.py:211-216)
            tensors[pre + names[k]] = v
            deq[k] = v
        else:
            arr, raw = stored(v, dtype, seed=seed + 10 + i)
            tensors[pre + names[k]] = (arr, raw)
            deq[k] = dequantized(arr, raw).reshape(v.shape)
    write(path, tensors, {"meshdec.resolution": 256, "sam3d.dtype": dtype}, arch="sam3d.meshdec")
    return deq, pre


@pytest.mark.parametrize("prec,tol", PRECS)
@pytest.mark.parametrize("dtype", ["f32", "f16", "q8_0", "q4_0", "q4_1", "q4_k"])
def test_mesh_level_from_gguf(ctx, tmp_path, prec, tol, dtype):
    cin, cout = 192, 96
    path = str(tmp_path / f"slat_decoder_mesh-{dtype}.gguf")
    p, pre = mesh_level_gguf(path, cin, cout, dtype, seed=30)
    g = s3dsp.Gguf(path)
    assert g.str("sam3d.dtype") == dtype
    parents = workloads.ellipsoid_shell(24, 5)
    np_ = len(parents)
    x = workloads.normal((np_, cin), 12)
    cc_exp, nb = oracle.mesh_subdivide(parents)
    exp = oracle.mesh_upsample_level(x, nb, p)
    w1 = g.load_weights(ctx, pre + "out_layers.0.conv.weight", s3dsp.LAYOUT_MESH_PACKED, 27, cin, cout, prec)
    w2 = g.load_weights(ctx, pre + "out_layers.3.conv.weight", s3dsp.LAYOUT_MESH_PACKED, 27, cout, cout, prec)
    ws = g.load_weights(ctx, pre + "skip_connection.conv.weight", s3dsp.LAYOUT_MESH_PACKED, 1, cin, cout, prec)
    v = {k: g.load(ctx, pre + k) for k in ("act_layers.0.weight", "act_layers.0.bias", "out_layers.0.conv.bias",
                                           "out_layers.1.weight", "out_layers.1.bias", "out_layers.3.conv.bias",
                                           "skip_connection.conv.bias")}
    hp = ctx.hash_build(torch.from_numpy(parents).cuda(), reject_duplicates=True)
    cc = torch.empty((8 * np_, 4), dtype=torch.int32, device="cuda")
    out = torch.empty((8 * np_, cout), device="cuda")
    ctx.mesh_upsample_level(hp, prec, torch.from_numpy(x).cuda(), cout, v["act_layers.0.weight"],
                            v["act_layers.0.bias"], w1, v["out_layers.0.conv.bias"], v["out_layers.1.weight"],
                            v["out_layers.1.bias"], w2, v["out_layers.3.conv.bias"], ws,
                            v["skip_connection.conv.bias"], cc, out)
    torch.cuda.synchronize()
    assert np.array_equal(cc.cpu().numpy(), cc_exp)
    gate(rel_l2(out.cpu().numpy(), exp), tol)


def test_weight_shape_checked(ctx, tmp_path):
    path = str(tmp_path / "m.gguf")
    _, pre = mesh_level_gguf(path, 64, 32, "f16", seed=40)
    g = s3dsp.Gguf(path)
    # the packed layout stores cout*cin as one extent: a wrong channel count or kernel volume is caught
    with pytest.raises(s3dsp.S3dError, match="layout wants"):
        g.load_weights(ctx, pre + "out_layers.0.conv.weight", s3dsp.LAYOUT_MESH_PACKED, 27, 48, 32,
                       s3dsp.PREC_BF16)
    with pytest.raises(s3dsp.S3dError, match="layout wants"):
        g.load_weights(ctx, pre + "out_layers.0.conv.weight", s3dsp.LAYOUT_MESH_PACKED, 1, 64, 32,
                       s3dsp.PREC_BF16)
    with pytest.raises(s3dsp.S3dError, match="not in"):
        g.load_weights(ctx, "meshdec.nothing.weight", s3dsp.LAYOUT_LINEAR, 1, 64, 32, s3dsp.PREC_BF16)
