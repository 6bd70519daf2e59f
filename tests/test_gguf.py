"""GGUF / SAMT parsing through the C-ABI (no GPU): tensor directory, raw
bytes and metadata against gguf-py's reader; SAMT round trips and the
reference's shipped SAMT fixture; malformed files rejected."""
import os

import numpy as np
import pytest
import gguf

import s3dsp
from gguf_fixtures import QTYPES, stored, write

# the reference tree (read only when present; the same variable __graft_entry__.build() reads)
REFERENCE_ROOT = os.environ.get("S3D_REFERENCE_ROOT", "/root/reference")
REF_SAMT = os.path.join(REFERENCE_ROOT, "tests", "objects_runtime", "fixtures", "ss_occ_f32.samt")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture()
def sample(tmp_path):
    rng = np.random.default_rng(1)
    tensors = {"bias": rng.normal(size=96).astype(np.float32),
               "ids": (np.arange(12, dtype=np.int32).reshape(3, 4), None)}
    for i, dt in enumerate(QTYPES):
        tensors[f"w.{dt}"] = stored(rng.normal(size=(3, 512)).astype(np.float32), dt, seed=i)
    kv = {"meshdec.resolution": 256, "meshdec.mlp_ratio": 4.0, "meshdec.attn_mode": "swin",
          "cemb.groups": [3, 1, 4, 1, 5], "names": ["alpha", "", "gamma"], "flag": True}
    path = str(tmp_path / "sample.gguf")
    write(path, tensors, kv)
    return path


def test_directory_and_bytes_match_gguf_py(sample):
    g = s3dsp.Gguf(sample)
    r = gguf.GGUFReader(sample)
    assert g.names() == [t.name for t in r.tensors]
    for t in r.tensors:
        inf = g.info(t.name)
        assert inf["type"] == int(t.tensor_type), t.name
        assert inf["shape"] == tuple(int(v) for v in reversed(t.shape)), t.name
        assert inf["nbytes"] == int(t.n_bytes), t.name
        assert np.array_equal(g.read(t.name), np.frombuffer(t.data.tobytes(), np.uint8)), t.name


def test_metadata(sample):
    g = s3dsp.Gguf(sample)
    assert g.u32("meshdec.resolution") == 256 and g.i32("meshdec.resolution") == 256
    assert g.f32("meshdec.mlp_ratio") == 4.0
    assert g.str("meshdec.attn_mode") == "swin"
    assert g.str("general.architecture") == "sam3d.test"
    assert g.i32_array("cemb.groups") == [3, 1, 4, 1, 5]
    assert g.str_array("names") == ["alpha", "", "gamma"]
    # defaults for missing keys and for keys of another type (GGUFModel semantics)
    assert g.u32("missing", 9) == 9 and g.f32("meshdec.resolution", -1.0) == -1.0
    assert g.str("meshdec.resolution", "d") == "d" and g.i32_array("names") == []
    with pytest.raises(KeyError):
        g.info("nope")


@pytest.mark.parametrize("damage", ["magic", "version", "truncated", "empty"])
def test_malformed_rejected(sample, tmp_path, damage):
    data = bytearray(open(sample, "rb").read())
    if damage == "magic":
        data[0:4] = b"GGUX"
    elif damage == "version":
        data[4:8] = (9).to_bytes(4, "little")
    elif damage == "truncated":
        data = data[: len(data) // 2]
    else:
        data = bytearray()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(bytes(data))
    with pytest.raises(s3dsp.S3dError):
        s3dsp.Gguf(str(bad))


def test_samt_round_trip(tmp_path):
    x = np.random.default_rng(2).normal(size=(5, 7, 3)).astype(np.float32)
    p = str(tmp_path / "x.samt")
    s3dsp.samt_write(p, x)
    y, inf = s3dsp.samt_read(p)
    assert inf["type"] == s3dsp.GGML_F32 and y.shape == x.shape and np.array_equal(x, y)
    ids = np.arange(10, dtype=np.int32).reshape(2, 5)
    s3dsp.samt_write(p, ids)
    z, inf = s3dsp.samt_read(p)
    assert inf["type"] == s3dsp.GGML_I32 and np.array_equal(z, ids)
    # writers that used type id 30 for int32 read back as I32 (common.cpp:108-110)
    s3dsp.samt_write(p, ids, ggml_type=30)
    z, inf = s3dsp.samt_read(p)
    assert inf["type"] == s3dsp.GGML_I32 and np.array_equal(z, ids)
    # byte layout: magic, ndims, ne (fastest first), type, data
    raw = open(p, "rb").read()
    assert raw[:4] == b"SAMT" and int.from_bytes(raw[4:8], "little") == 2
    assert int.from_bytes(raw[8:16], "little") == 5 and int.from_bytes(raw[16:24], "little") == 2


def test_samt_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.samt"
    p.write_bytes(b"SAMX" + bytes(20))
    with pytest.raises(s3dsp.S3dError):
        s3dsp.samt_read(str(p))
    p.write_bytes(b"SAMT" + (9).to_bytes(4, "little"))
    with pytest.raises(s3dsp.S3dError):
        s3dsp.samt_read(str(p))


@pytest.mark.skipif(not os.path.exists(REF_SAMT), reason="reference tree not present")
def test_reads_the_reference_samt_fixture():
    """The reference's real 64^3 SS-decoder output: shape and the occupancy
    bitmask recorded in tests/golden/ss_occ_mask.npz."""
    x, inf = s3dsp.samt_read(REF_SAMT)
    assert inf["type"] == s3dsp.GGML_F32 and x.shape == (64, 64, 64)
    bits = np.load(os.path.join(GOLDEN, "ss_occ_mask.npz"))["bits"]
    # SAMT ne = (64, 64, 64) fastest first; the fixture's flat order is (x*64 + y)*64 + z
    assert np.array_equal(np.packbits((x.reshape(-1) > 0)), bits)
