"""The C-ABI library loads without a GPU and exports every declared symbol."""
import ctypes
import os
import re

import s3dsp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for hdr in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not hdr.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", hdr)).read()
        names += re.findall(r"S3DSP_API\s+[\w\s\*]+?\b(s3dsp_\w+)\s*\(", text)
    return names


def test_header_declares_expected_surface():
    names = declared_symbols()
    assert len(names) == len(set(names))
    assert sorted(names) == sorted(s3dsp.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(s3dsp.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_cpu_only_entry_points():
    """Pure host helpers answer without touching a GPU."""
    L = s3dsp.load()
    assert L.s3dsp_abi_version() == 1
    # bf16 packing: [27][cout_pad16][cin_pad64]; f32: [27][cin_pad16][cout_pad64]
    assert L.s3dsp_weights_packed_bytes(s3dsp.PREC_BF16, 27, 96, 101) == 27 * 112 * 128 * 2
    assert L.s3dsp_weights_packed_bytes(s3dsp.PREC_F32_STRICT, 27, 96, 101) == 27 * 96 * 128 * 4
    assert L.s3dsp_gn_partials_count(15159, 256, 32) == 119 * 32 * 2


def test_context_create_reports_errors_through_the_buffer():
    """With no usable device the call fails with a status and a message, never
    a crash (the reference's error-buffer convention, include/sam3d.h:32-34)."""
    L = s3dsp.load()
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(256)
    st = L.s3dsp_context_create(9999, None, 0, ctypes.byref(h), buf, 256)
    assert st != s3dsp.S3D_OK and h.value is None and len(buf.value) > 0
    # NULL,0 discards diagnostics
    st = L.s3dsp_context_create(9999, None, 0, ctypes.byref(h), None, 0)
    assert st != s3dsp.S3D_OK
