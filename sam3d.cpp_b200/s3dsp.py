"""Python front-end of libs3dsp.so (the C-ABI CUDA library), via ctypes.

This is the host-side mirror of the reference's internal C++ surface for the
sparse-convolution path (src/objects_runtime/sparse_ops.hpp table builders,
mesh_decoder_graph.cpp / slat_flow_graph.cpp graph pieces, session.cpp
decode_object_mesh). Device memory is owned by the caller (torch tensors are
the convenient allocator here); the library never falls back to the CPU: if
libs3dsp.so is missing or no sm_100 GPU is present, every entry point raises.

Error handling mirrors the reference C API (include/sam3d.h:20-40): each call
returns an s3d_status and fills an error buffer; non-zero statuses raise
S3dError carrying both.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libs3dsp.so")

S3D_OK, S3D_INVALID_ARGUMENT, S3D_OUT_OF_MEMORY, S3D_INTERNAL_ERROR = 0, 1, 2, 3
F32, BF16, F16 = 0, 1, 2
PREC_F32_STRICT, PREC_BF16, PREC_F32_3XTF32 = 0, 1, 2
LAYOUT_SLAT_ROW, LAYOUT_MESH_PACKED, LAYOUT_LINEAR, LAYOUT_SPCONV_1X1, LAYOUT_TRANSPOSED_2X2X2 = 0, 1, 2, 3, 4
SENTINEL_SLAT_N, SENTINEL_MESH_NEG1 = 0, 1
EPI_SILU, PRO_AFFINE_SILU, CONV_CTA_PAIR, CONV_TILE128, CONV_STREAM_K, CONV_STREAM_K128, EPI_GELU = 1, 2, 4, 8, 16, 32, 64
CONV_SPLIT_PAIRS = 128
CONV_HALO = 256
CONTEXT_DEFERRED_CHECKS = 1
CONTEXT_OWN_STREAM = 2
CONTEXT_COPY_STREAMS = 4

# every symbol include/s3dsp.h declares (tests check the library exports them)
EXPORTED = [
    "s3dsp_abi_version", "s3dsp_context_create", "s3dsp_context_free", "s3dsp_context_stream", "s3dsp_context_set_sm_limit",
    "s3dsp_context_check", "s3dsp_context_fork", "s3dsp_context_join", "s3dsp_memory_stats", "s3dsp_device_alloc", "s3dsp_device_free", "s3dsp_copy_to_device",
    "s3dsp_copy_to_host", "s3dsp_hash_build", "s3dsp_hash_free", "s3dsp_hash_size",
    "s3dsp_hash_lookup", "s3dsp_gs_window_tables", "s3dsp_ape", "s3dsp_gather_rows", "s3dsp_window_attention", "s3dsp_flexicubes_tables_create",
    "s3dsp_flexicubes_tables_free", "s3dsp_flexicubes_extract", "s3dsp_mesh_info", "s3dsp_mesh_device", "s3dsp_mesh_copy",
    "s3dsp_mesh_free", "s3dsp_gguf_open", "s3dsp_gguf_close", "s3dsp_gguf_n_tensors", "s3dsp_gguf_find",
    "s3dsp_gguf_tensor_info", "s3dsp_gguf_u32", "s3dsp_gguf_i32", "s3dsp_gguf_f32", "s3dsp_gguf_str",
    "s3dsp_gguf_array_len", "s3dsp_gguf_str_array", "s3dsp_gguf_i32_array", "s3dsp_gguf_read", "s3dsp_gguf_load",
    "s3dsp_gguf_load_weights", "s3dsp_dequantize", "s3dsp_samt_info", "s3dsp_samt_read", "s3dsp_samt_write",
    "s3dsp_shard_plan_morton", "s3dsp_shard_info", "s3dsp_shard_lists", "s3dsp_shard_free", "s3dsp_nccl_unique_id",
    "s3dsp_nccl_comm_create", "s3dsp_nccl_comm_free", "s3dsp_halo_exchange", "s3dsp_occupancy_coords", "s3dsp_prune_surface", "s3dsp_downsample_coords",
    "s3dsp_kmap_build_subm3", "s3dsp_kmap_build_subm3_rows", "s3dsp_kmap_build_subm3_range", "s3dsp_subdivide", "s3dsp_kmap_free",
    "s3dsp_kmap_rows", "s3dsp_kmap_export_dense", "s3dsp_kmap_pairs", "s3dsp_kmap_pairs_noalloc",
    "s3dsp_weights_packed_bytes", "s3dsp_weights_pack", "s3dsp_gn_partials_count", "s3dsp_conv", "s3dsp_conv_concat",
    "s3dsp_conv_kernel", "s3dsp_conv_kernel_shift", "s3dsp_layer_norm_concat", "s3dsp_kmap_compose", "s3dsp_slat_res_block_concat",
    "s3dsp_gn_stats", "s3dsp_gn_finalize", "s3dsp_channel_affine", "s3dsp_layer_norm",
    "s3dsp_convert", "s3dsp_slat_tables_build", "s3dsp_slat_tables_free", "s3dsp_slat_tables_coarse_rows",
    "s3dsp_slat_tables_coarse_kmap", "s3dsp_slat_tables_export", "s3dsp_slat_downsample", "s3dsp_slat_upsample",
    "s3dsp_res_block_gn", "s3dsp_mesh_upsample_level", "s3dsp_slat_res_block", "s3dsp_res_block_gn_host", "s3dsp_res_block_gn_host_queued",
    "s3dsp_mesh_upsample_level_host",
]


class S3dError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"s3d_status {status}: {message}")
        self.status = status
        self.message = message


_lib = None
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_cp = ctypes.c_char_p
_f = ctypes.c_float


def load(path: str = LIB_PATH):
    """Load libs3dsp.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built (run __graft_entry__.build())")
    L = ctypes.CDLL(path)
    sig = {
        "s3dsp_abi_version": (_u32, []),
        "s3dsp_context_create": (_u32, [_i32, _vp, _u32, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_context_free": (None, [_vp]),
        "s3dsp_context_stream": (_vp, [_vp]),
        "s3dsp_context_set_sm_limit": (_u32, [_vp, _i32, _cp, _u64]),
        "s3dsp_context_check": (_u32, [_vp, _cp, _u64]),
        "s3dsp_context_fork": (_u32, [_vp, _cp, _u64]),
        "s3dsp_context_join": (_u32, [_vp, _cp, _u64]),
        "s3dsp_device_alloc": (_u32, [_vp, _u64, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_device_free": (None, [_vp, _vp]),
        "s3dsp_copy_to_device": (_u32, [_vp, _vp, _vp, _u64, _cp, _u64]),
        "s3dsp_copy_to_host": (_u32, [_vp, _vp, _vp, _u64, _cp, _u64]),
        "s3dsp_memory_stats": (_u32, [_i32, ctypes.POINTER(_u64), ctypes.POINTER(_u64), ctypes.POINTER(_u64), _i32,
                                      _cp, _u64]),
        "s3dsp_hash_build": (_u32, [_vp, _vp, _i64, _i32, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_hash_free": (None, [_vp, _vp]),
        "s3dsp_hash_size": (_i64, [_vp]),
        "s3dsp_hash_lookup": (_u32, [_vp, _vp, _vp, _i64, _vp, _cp, _u64]),
        "s3dsp_gs_window_tables": (_u32, [_vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _i64, ctypes.POINTER(_i64), _cp,
                                          _u64]),
        "s3dsp_ape": (_u32, [_vp, _vp, _i64, _i32, _vp, _cp, _u64]),
        "s3dsp_gather_rows": (_u32, [_vp, _vp, _u32, _i64, _i64, _vp, _i64, _vp, _u32, _cp, _u64]),
        "s3dsp_window_attention": (_u32, [_vp, _vp, _i64, _i64, _i32, _vp, _i64, _vp, _vp, _cp, _u64]),
        "s3dsp_flexicubes_tables_create": (_u32, [_vp, _vp, _vp, _vp, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_flexicubes_tables_free": (None, [_vp, _vp]),
        "s3dsp_flexicubes_extract": (_u32, [_vp, _vp, _vp, _vp, _i64, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_mesh_info": (_u32, [_vp] + [ctypes.POINTER(_i64)] * 4),
        "s3dsp_mesh_device": (_u32, [_vp] + [ctypes.POINTER(_vp)] * 6),
        "s3dsp_mesh_copy": (_u32, [_vp, _vp] + [_vp] * 6 + [_cp, _u64]),
        "s3dsp_mesh_free": (None, [_vp, _vp]),
        "s3dsp_gguf_open": (_u32, [ctypes.c_char_p, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_gguf_close": (None, [_vp]),
        "s3dsp_gguf_n_tensors": (_i64, [_vp]),
        "s3dsp_gguf_find": (_i64, [_vp, ctypes.c_char_p]),
        "s3dsp_gguf_tensor_info": (_u32, [_vp, _i64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i32),
                                          ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(_u64)]),
        "s3dsp_gguf_u32": (ctypes.c_uint32, [_vp, ctypes.c_char_p, ctypes.c_uint32]),
        "s3dsp_gguf_i32": (_i32, [_vp, ctypes.c_char_p, _i32]),
        "s3dsp_gguf_f32": (ctypes.c_float, [_vp, ctypes.c_char_p, ctypes.c_float]),
        "s3dsp_gguf_str": (_i64, [_vp, ctypes.c_char_p, _cp, _u64]),
        "s3dsp_gguf_array_len": (_i64, [_vp, ctypes.c_char_p]),
        "s3dsp_gguf_str_array": (_i64, [_vp, ctypes.c_char_p, _i64, _cp, _u64]),
        "s3dsp_gguf_i32_array": (_i64, [_vp, ctypes.c_char_p, _vp, _i64]),
        "s3dsp_gguf_read": (_u32, [_vp, _i64, _vp, _u64, _cp, _u64]),
        "s3dsp_gguf_load": (_u32, [_vp, _vp, _i64, _u32, _vp, _i64, _cp, _u64]),
        "s3dsp_gguf_load_weights": (_u32, [_vp, _vp, ctypes.c_char_p, _u32, _i32, _i64, _i64, _u32, _vp, _cp, _u64]),
        "s3dsp_dequantize": (_u32, [_vp, _i32, _vp, _i64, _u32, _vp, _cp, _u64]),
        "s3dsp_samt_info": (_u32, [ctypes.c_char_p, ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(_i32),
                                   ctypes.POINTER(_u64), _cp, _u64]),
        "s3dsp_samt_read": (_u32, [ctypes.c_char_p, _vp, _u64, _cp, _u64]),
        "s3dsp_samt_write": (_u32, [ctypes.c_char_p, _i32, _vp, _i32, _vp, _u64, _cp, _u64]),
        "s3dsp_shard_plan_morton": (_u32, [_vp, _i64, _i32, _i32, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_shard_info": (_u32, [_vp] + [ctypes.POINTER(_i64)] * 4),
        "s3dsp_shard_lists": (_u32, [_vp] + [_vp] * 5),
        "s3dsp_shard_free": (None, [_vp, _vp]),
        "s3dsp_nccl_unique_id": (_u32, [_vp, _cp, _u64]),
        "s3dsp_nccl_comm_create": (_u32, [_vp, _i32, _i32, _vp, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_nccl_comm_free": (None, [_vp]),
        "s3dsp_halo_exchange": (_u32, [_vp, _vp, _vp, _vp, _i64, _u32, _cp, _u64]),
        "s3dsp_occupancy_coords": (_u32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _i64, ctypes.POINTER(_i64), _cp,
                                          _u64]),
        "s3dsp_prune_surface": (_u32, [_vp, _vp, _i64, _i32, _vp, _i64, ctypes.POINTER(_i64), _cp, _u64]),
        "s3dsp_downsample_coords": (_u32, [_vp, _vp, _i64, _i64, _i32, ctypes.c_uint32, _vp, _i64,
                                           ctypes.POINTER(_i64), _cp, _u64]),
        "s3dsp_kmap_build_subm3": (_u32, [_vp, _vp, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_kmap_build_subm3_rows": (_u32, [_vp, _vp, _i64, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_kmap_build_subm3_range": (_u32, [_vp, _vp, _i64, _i64, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_subdivide": (_u32, [_vp, _vp, _vp, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_kmap_free": (None, [_vp, _vp]),
        "s3dsp_kmap_rows": (_i64, [_vp]),
        "s3dsp_kmap_export_dense": (_u32, [_vp, _vp, _u32, _vp, _cp, _u64]),
        "s3dsp_kmap_pairs": (_u32, [_vp, _vp, _vp, _vp, _i64, ctypes.POINTER(_i64), _cp, _u64]),
        "s3dsp_kmap_pairs_noalloc": (_u32, [_vp, _vp, _vp, _vp, _i64, ctypes.POINTER(_i64), _cp, _u64]),
        "s3dsp_weights_packed_bytes": (_i64, [_u32, _i32, _i64, _i64]),
        "s3dsp_weights_pack": (_u32, [_vp, _vp, _u32, _i32, _u32, _i32, _i64, _i64, _u32, _vp, _cp, _u64]),
        "s3dsp_gn_partials_count": (_i64, [_i64, _i64, _i32]),
        "s3dsp_conv_kernel": (_cp, [_vp, _i64, _i32, _i64, _i64, _u32, _u32]),
        "s3dsp_conv_kernel_shift": (_cp, [_vp, _i64, _i32, _i64, _i64, _i32, _u32, _u32]),
        "s3dsp_conv": (_u32, [_vp, _vp, _i32, _u32, _vp, _u32, _i64, _i64, _i32, _vp, _vp, _vp, _u32, _i32,
                              _vp, _u32, _i64, _i64, _u32, _vp, _vp, _vp, _vp, _i32, _cp, _u64]),
        "s3dsp_conv_concat": (_u32, [_vp, _vp, _i32, _u32, _vp, _i64, _vp, _i64, _u32, _i64, _i32, _vp, _vp, _vp,
                                     _u32, _i32, _vp, _u32, _i64, _i64, _u32, _vp, _vp, _vp, _vp, _i32, _cp, _u64]),
        "s3dsp_layer_norm_concat": (_u32, [_vp, _vp, _i64, _vp, _i64, _u32, _i64, _f, _vp, _vp, _vp, _vp, _i32, _vp,
                                           _u32, _cp, _u64]),
        "s3dsp_kmap_compose": (_u32, [_vp, _vp, _vp, _i64, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_slat_res_block_concat": (_u32, [_vp, _vp, _vp, _u32, _vp, _i64, _vp, _i64, _i64, _i64] + [_vp] * 11
                                        + [_cp, _u64]),
        "s3dsp_gn_stats": (_u32, [_vp, _vp, _u32, _i64, _i64, _i32, _vp, _cp, _u64]),
        "s3dsp_gn_finalize": (_u32, [_vp, _vp, _i64, _i64, _i32, _f, _vp, _vp, _vp, _vp, _vp, _cp, _u64]),
        "s3dsp_channel_affine": (_u32, [_vp, _vp, _u32, _i64, _i64, _vp, _vp, _vp, _i32, _vp, _u32, _cp, _u64]),
        "s3dsp_layer_norm": (_u32, [_vp, _vp, _u32, _i64, _i64, _f, _vp, _vp, _vp, _vp, _i32, _vp, _u32, _cp,
                                    _u64]),
        "s3dsp_convert": (_u32, [_vp, _vp, _u32, _vp, _u32, _i64, _cp, _u64]),
        "s3dsp_slat_tables_build": (_u32, [_vp, _vp, ctypes.POINTER(_vp), _cp, _u64]),
        "s3dsp_slat_tables_free": (None, [_vp, _vp]),
        "s3dsp_slat_tables_coarse_rows": (_i64, [_vp]),
        "s3dsp_slat_tables_coarse_kmap": (_vp, [_vp]),
        "s3dsp_slat_tables_export": (_u32, [_vp, _vp, _vp, _vp, _vp, _vp, _cp, _u64]),
        "s3dsp_slat_downsample": (_u32, [_vp, _vp, _vp, _u32, _i64, _vp, _u32, _cp, _u64]),
        "s3dsp_slat_upsample": (_u32, [_vp, _vp, _vp, _u32, _i64, _vp, _u32, _cp, _u64]),
        "s3dsp_res_block_gn": (_u32, [_vp, _vp, _u32, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _f, _vp,
                                      _cp, _u64]),
        "s3dsp_mesh_upsample_level": (_u32, [_vp, _vp, _u32, _vp, _i64, _i64] + [_vp] * 12 + [_cp, _u64]),
        "s3dsp_slat_res_block": (_u32, [_vp, _vp, _u32, _vp, _i64, _i64, _i64] + [_vp] * 11 + [_cp, _u64]),
        "s3dsp_res_block_gn_host": (_u32, [_vp, _u32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _f,
                                           _vp, _cp, _u64]),
        "s3dsp_res_block_gn_host_queued": (_u32, [_vp, _u32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                                  _i32, _f, _vp, _cp, _u64]),
        "s3dsp_mesh_upsample_level_host": (_u32, [_vp, _u32, _vp, _i64, _vp, _i64, _i64] + [_vp] * 12 + [_cp, _u64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _call(fn, *args):
    buf = ctypes.create_string_buffer(512)
    st = fn(*args, buf, ctypes.c_uint64(len(buf)))
    if st != S3D_OK:
        raise S3dError(st, buf.value.decode(errors="replace"))


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor, or None."""
    if t is None:
        return None
    return t.data_ptr()


def dtype_code(t) -> int:
    import torch
    return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}[t.dtype]


class Kmap:
    def __init__(self, ctx: "Context", handle: int, rows: int):
        self.ctx, self.handle, self.rows = ctx, handle, rows

    def free(self):
        if self.handle:
            load().s3dsp_kmap_free(self.ctx.handle, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Hash:
    def __init__(self, ctx: "Context", handle: int, n: int):
        self.ctx, self.handle, self.n = ctx, handle, n

    def free(self):
        if self.handle:
            load().s3dsp_hash_free(self.ctx.handle, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class SlatTables:
    def __init__(self, ctx: "Context", handle: int, nf: int):
        self.ctx, self.handle, self.nf = ctx, handle, nf
        self.nc = load().s3dsp_slat_tables_coarse_rows(handle)
        self.coarse_kmap = Kmap(ctx, None, self.nc)
        self.coarse_kmap.handle = load().s3dsp_slat_tables_coarse_kmap(handle)
        self.coarse_kmap.free = lambda: None  # owned by the tables

    def free(self):
        if self.handle:
            load().s3dsp_slat_tables_free(self.ctx.handle, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class FlexiCubesTables:
    def __init__(self, ctx: "Context", handle: int):
        self.ctx, self.handle = ctx, handle

    def free(self):
        if self.handle:
            load().s3dsp_flexicubes_tables_free(self.ctx.handle, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Mesh:
    """A device mesh from s3dsp_flexicubes_extract (counts + host copies)."""

    def __init__(self, ctx: "Context", handle: int):
        self.ctx, self.handle = ctx, handle
        c = [_i64() for _ in range(4)]
        st = load().s3dsp_mesh_info(handle, *(ctypes.byref(v) for v in c))
        if st != S3D_OK:
            raise S3dError(st, "s3dsp_mesh_info")
        self.n_vertices, self.n_faces, self.n_surface, self.n_edges = (v.value for v in c)

    def host(self) -> dict:
        """dict(vertices [V, 3], attrs [V, 6], faces [F, 3], surface [S],
        cases [S], edges [E, 2]) as numpy arrays."""
        import numpy as np
        out = dict(vertices=np.zeros((self.n_vertices, 3), np.float32),
                   attrs=np.zeros((self.n_vertices, 6), np.float32),
                   faces=np.zeros((self.n_faces, 3), np.int32), surface=np.zeros(self.n_surface, np.int32),
                   cases=np.zeros(self.n_surface, np.int32), edges=np.zeros((self.n_edges, 2), np.int32))
        _call(load().s3dsp_mesh_copy, self.ctx.handle, self.handle,
              *(out[k].ctypes.data for k in ("vertices", "attrs", "faces", "surface", "cases", "edges")))
        return out

    def free(self):
        if self.handle:
            load().s3dsp_mesh_free(self.ctx.handle, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0, GGML_Q4_K, GGML_I32, GGML_BF16 = 0, 1, 2, 3, 8, 12, 26, 30


class Gguf:
    """A GGUF weight file (s3dsp_gguf_*): metadata and tensor directory on the
    host; tensors read raw or loaded to the device (dequantised / packed).
    Shapes are numpy order (ne reversed)."""

    def __init__(self, path: str):
        h = _vp()
        _call(load().s3dsp_gguf_open, path.encode(), ctypes.byref(h))
        self.handle = h.value
        self.path = path

    def close(self):
        if getattr(self, "handle", None):
            load().s3dsp_gguf_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list:
        L = load()
        out = []
        for i in range(L.s3dsp_gguf_n_tensors(self.handle)):
            nm = ctypes.c_char_p()
            L.s3dsp_gguf_tensor_info(self.handle, i, ctypes.byref(nm), None, None, None, None)
            out.append(nm.value.decode())
        return out

    def index(self, name: str) -> int:
        i = load().s3dsp_gguf_find(self.handle, name.encode())
        if i < 0:
            raise KeyError(name)
        return i

    def info(self, name: str) -> dict:
        t, nd, nb = _i32(), _i32(), _u64()
        ne = (_i64 * 4)()
        st = load().s3dsp_gguf_tensor_info(self.handle, self.index(name), None, ctypes.byref(t), ctypes.byref(nd), ne,
                                           ctypes.byref(nb))
        if st != S3D_OK:
            raise S3dError(st, "s3dsp_gguf_tensor_info")
        return dict(type=t.value, shape=tuple(reversed(ne[:nd.value])), nbytes=nb.value)

    def u32(self, key, default=0):
        return load().s3dsp_gguf_u32(self.handle, key.encode(), default)

    def i32(self, key, default=0):
        return load().s3dsp_gguf_i32(self.handle, key.encode(), default)

    def f32(self, key, default=0.0):
        return load().s3dsp_gguf_f32(self.handle, key.encode(), default)

    def str(self, key, default=""):
        n = load().s3dsp_gguf_str(self.handle, key.encode(), None, 0)
        if n < 0:
            return default
        buf = ctypes.create_string_buffer(n + 1)
        load().s3dsp_gguf_str(self.handle, key.encode(), buf, n + 1)
        return buf.raw[:n].decode()

    def str_array(self, key) -> list:
        L = load()
        n = L.s3dsp_gguf_array_len(self.handle, key.encode())
        out = []
        for i in range(max(n, 0)):
            m = L.s3dsp_gguf_str_array(self.handle, key.encode(), i, None, 0)
            if m < 0:
                return []
            buf = ctypes.create_string_buffer(m + 1)
            L.s3dsp_gguf_str_array(self.handle, key.encode(), i, buf, m + 1)
            out.append(buf.raw[:m].decode())
        return out

    def i32_array(self, key) -> list:
        import numpy as np
        n = load().s3dsp_gguf_i32_array(self.handle, key.encode(), None, 0)
        if n < 0:
            return []
        a = np.zeros(n, np.int32)
        load().s3dsp_gguf_i32_array(self.handle, key.encode(), a.ctypes.data, n)
        return a.tolist()

    def read(self, name: str):
        """Raw stored bytes (numpy uint8)."""
        import numpy as np
        a = np.zeros(self.info(name)["nbytes"], np.uint8)
        _call(load().s3dsp_gguf_read, self.handle, self.index(name), a.ctypes.data, a.nbytes)
        return a

    def load(self, ctx: "Context", name: str, bf16: bool = False):
        """A float tensor on ctx's device as f32 (or bf16), numpy-order shape."""
        import torch
        shape = self.info(name)["shape"]
        out = torch.empty(shape, dtype=torch.bfloat16 if bf16 else torch.float32, device=f"cuda:{ctx.device}")
        _call(load().s3dsp_gguf_load, ctx.handle, self.handle, self.index(name), BF16 if bf16 else F32, ptr(out),
              out.numel())
        return out

    def load_weights(self, ctx: "Context", name: str, layout: int, kvol: int, cin: int, cout: int, precision: int):
        """A conv / linear weight packed for `precision` (uint8 device buffer)."""
        import torch
        dst = torch.empty(Context.packed_bytes(precision, kvol, cin, cout), dtype=torch.uint8,
                          device=f"cuda:{ctx.device}")
        _call(load().s3dsp_gguf_load_weights, ctx.handle, self.handle, name.encode(), layout, kvol, cin, cout,
              precision, ptr(dst))
        return dst


class ShardPlan:
    """s3dsp_shard_plan_morton: the Morton-slab plan of one rank, with its
    lists as numpy arrays (own, ghost, recv_counts, send_counts, send_rows)."""

    def __init__(self, coords, world: int, rank: int):
        import numpy as np
        c = np.ascontiguousarray(coords, dtype=np.int32).reshape(-1, 4)
        h = _vp()
        _call(load().s3dsp_shard_plan_morton, c.ctypes.data, c.shape[0], world, rank, ctypes.byref(h))
        self.handle, self.world, self.rank = h.value, world, rank
        no, ni, ng, ns = (_i64() for _ in range(4))
        load().s3dsp_shard_info(self.handle, ctypes.byref(no), ctypes.byref(ni), ctypes.byref(ng), ctypes.byref(ns))
        self.n_own, self.n_interior, self.n_ghost = no.value, ni.value, ng.value
        self.own = np.zeros(no.value, np.int64)
        self.ghost = np.zeros(ng.value, np.int64)
        self.recv_counts = np.zeros(world, np.int64)
        self.send_counts = np.zeros(world, np.int64)
        self.send_rows = np.zeros(ns.value, np.int64)
        load().s3dsp_shard_lists(self.handle, *(a.ctypes.data for a in (self.own, self.ghost, self.recv_counts,
                                                                         self.send_counts, self.send_rows)))

    def free(self, ctx: "Context | None" = None):
        if getattr(self, "handle", None):
            load().s3dsp_shard_free(ctx.handle if ctx else None, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _call(load().s3dsp_nccl_unique_id, ctypes.cast(buf, ctypes.c_void_p))
    return buf.raw


def memory_stats(device: int = 0, reset_high: bool = False) -> dict:
    """Bytes the library's own device pool holds on `device`: reserved, in use
    and the high-water mark of use (reset to the current use afterwards when
    reset_high)."""
    r, u, h = _u64(), _u64(), _u64()
    _call(load().s3dsp_memory_stats, device, ctypes.byref(r), ctypes.byref(u), ctypes.byref(h), int(reset_high))
    return {"reserved": r.value, "used": u.value, "used_high": h.value}


def samt_info(path: str) -> dict:
    nd, t, nb = _i32(), _i32(), _u64()
    ne = (_i64 * 8)()
    _call(load().s3dsp_samt_info, path.encode(), ctypes.byref(nd), ne, ctypes.byref(t), ctypes.byref(nb))
    return dict(shape=tuple(reversed(ne[:nd.value])), type=t.value, nbytes=nb.value)


def samt_read(path: str):
    """(raw bytes as numpy uint8, info dict); F32 / I32 tensors come back typed."""
    import numpy as np
    inf = samt_info(path)
    a = np.zeros(inf["nbytes"], np.uint8)
    _call(load().s3dsp_samt_read, path.encode(), a.ctypes.data, a.nbytes)
    if inf["type"] == GGML_F32:
        return a.view(np.float32).reshape(inf["shape"]), inf
    if inf["type"] == GGML_I32:
        return a.view(np.int32).reshape(inf["shape"]), inf
    return a, inf


def samt_write(path: str, array, ggml_type: int | None = None, shape=None):
    """Writes a numpy array (F32 / I32 inferred) or raw bytes with an explicit
    type and numpy-order shape."""
    import numpy as np
    a = np.ascontiguousarray(array)
    if ggml_type is None:
        ggml_type = {np.dtype(np.float32): GGML_F32, np.dtype(np.int32): GGML_I32}[a.dtype]
    shape = a.shape if shape is None else shape
    ne = (_i64 * len(shape))(*reversed(shape))
    _call(load().s3dsp_samt_write, path.encode(), len(shape), ne, ggml_type, a.ctypes.data, a.nbytes)


class Context:
    """One device + one CUDA stream (default: torch's current stream, so the
    library's kernels are ordered with torch's copies and events)."""

    def __init__(self, device: int = 0, stream: int | None = None, flags: int = 0):
        L = load()
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(device).cuda_stream
        h = _vp()
        _call(L.s3dsp_context_create, device, stream, flags, ctypes.byref(h))
        self.handle = h.value
        self.device = device
        self.flags = flags

    def close(self):
        if getattr(self, "handle", None):
            load().s3dsp_context_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self):
        _call(load().s3dsp_context_check, self.handle)

    def fork(self):
        """CONTEXT_COPY_STREAMS: order the copy streams after the context's stream."""
        _call(load().s3dsp_context_fork, self.handle)

    def join(self):
        """CONTEXT_COPY_STREAMS: order the context's stream after its copy streams."""
        _call(load().s3dsp_context_join, self.handle)

    def set_sm_limit(self, sms: int):
        """Size this context's SM-proportional grids for `sms` SMs (0: all)."""
        _call(load().s3dsp_context_set_sm_limit, self.handle, sms)

    # ---- coordinate hash / kernel maps --------------------------------------------------------
    def hash_build(self, coords, reject_duplicates: bool = False) -> Hash:
        h = _vp()
        _call(load().s3dsp_hash_build, self.handle, ptr(coords), coords.shape[0], int(reject_duplicates),
              ctypes.byref(h))
        return Hash(self, h.value, coords.shape[0])

    def hash_lookup(self, hsh: Hash, query, rows_out):
        _call(load().s3dsp_hash_lookup, self.handle, hsh.handle, ptr(query), query.shape[0], ptr(rows_out))

    # ---- GS decoder window tables ---------------------------------------------
    def gs_window_tables(self, coords, shift: int, bkt_idx, bwd_idx, window: int = 8):
        """Fills bkt_idx / bwd_idx (device int32 [n]); returns the buckets as a
        numpy [k, 3] array of {tokens per window, first row, windows}."""
        import numpy as np
        n = coords.shape[0]
        cap = max(n, 1)
        bk = np.zeros((cap, 3), np.int32)
        nb = ctypes.c_int64()
        _call(load().s3dsp_gs_window_tables, self.handle, ptr(coords), n, shift, window, ptr(bkt_idx), ptr(bwd_idx),
              bk.ctypes.data, cap, ctypes.byref(nb))
        return bk[:nb.value]

    def ape(self, coords, out):
        _call(load().s3dsp_ape, self.handle, ptr(coords), coords.shape[0], out.shape[1], ptr(out))

    # ---- several GPUs --------------------------------------------------------
    def nccl_comm(self, world: int, rank: int, uid: bytes) -> int:
        c = _vp()
        buf = ctypes.create_string_buffer(uid, 128)
        _call(load().s3dsp_nccl_comm_create, self.handle, world, rank, ctypes.cast(buf, ctypes.c_void_p),
              ctypes.byref(c))
        return c.value

    def halo_exchange(self, plan: ShardPlan, comm: int, x):
        """Fill x's ghost rows [n_own, n_own + n_ghost) from the peers (x on this device)."""
        _call(load().s3dsp_halo_exchange, self.handle, plan.handle, comm, ptr(x), x.shape[1], dtype_code(x))

    def gather_rows(self, x, rows, y):
        """y[i] = x[rows[i]] (rows: device int32 [len(y)]), with y's dtype."""
        _call(load().s3dsp_gather_rows, self.handle, ptr(x), dtype_code(x), x.shape[0], x.shape[1], ptr(rows),
              y.shape[0], ptr(y), dtype_code(y))

    def window_attention(self, qkv, heads: int, windows, out, scatter=None):
        """Swin window attention over qkv [n, 3c] f32 in bucket order; windows:
        device int32 [nw, 2] (first row, rows); row i to out[scatter[i]]."""
        _call(load().s3dsp_window_attention, self.handle, ptr(qkv), qkv.shape[0], qkv.shape[1] // 3, heads,
              ptr(windows), windows.shape[0], ptr(scatter), ptr(out))

    # ---- FlexiCubes extraction ---------------------------------------------
    def flexicubes_tables(self, dmc, num_dual, check) -> FlexiCubesTables:
        """DMC tables (numpy int8 [256, 4, 7], int8 [256], int16 [256, 5])."""
        import numpy as np
        dmc = np.ascontiguousarray(dmc, np.int8)
        num_dual = np.ascontiguousarray(num_dual, np.int8)
        check = np.ascontiguousarray(check, np.int16)
        assert dmc.size == 256 * 28 and num_dual.size == 256 and check.size == 256 * 5
        h = _vp()
        _call(load().s3dsp_flexicubes_tables_create, self.handle, dmc.ctypes.data, num_dual.ctypes.data,
              check.ctypes.data, ctypes.byref(h))
        return FlexiCubesTables(self, h.value)

    def flexicubes(self, tables: FlexiCubesTables, raw, coords) -> Mesh:
        """extract_object_mesh over device raw [n, 101] f32 and coords [n, 4] int32."""
        h = _vp()
        _call(load().s3dsp_flexicubes_extract, self.handle, tables.handle, ptr(raw), ptr(coords), coords.shape[0],
              ctypes.byref(h))
        return Mesh(self, h.value)

    # ---- coordinate pipeline -----------------------------------------------
    def occupancy_coords(self, occ, out, batch: int = 0) -> int:
        """Rows (batch, x, y, z) of the cells of occ [X, Y, Z] > 0 into out [cap, 4]; returns the count."""
        n = ctypes.c_int64()
        nx, ny, nz = occ.shape
        _call(load().s3dsp_occupancy_coords, self.handle, ptr(occ), nx, ny, nz, batch, ptr(out), out.shape[0],
              ctypes.byref(n))
        return n.value

    def prune_surface(self, coords, out, max_axis_dist: int = 1) -> int:
        n = ctypes.c_int64()
        _call(load().s3dsp_prune_surface, self.handle, ptr(coords), coords.shape[0], max_axis_dist, ptr(out),
              out.shape[0], ctypes.byref(n))
        return n.value

    def downsample_coords(self, coords, out, max_coords: int = 42000, factor: int = 2, seed: int = 42) -> int:
        n = ctypes.c_int64()
        _call(load().s3dsp_downsample_coords, self.handle, ptr(coords), coords.shape[0], max_coords, factor, seed,
              ptr(out), out.shape[0], ctypes.byref(n))
        return n.value

    def kmap_subm3(self, hsh: Hash) -> Kmap:
        k = _vp()
        _call(load().s3dsp_kmap_build_subm3, self.handle, hsh.handle, ctypes.byref(k))
        return Kmap(self, k.value, hsh.n)

    def kmap_subm3_rows(self, hsh: Hash, n_out: int) -> Kmap:
        """Submanifold map of the hash's first n_out rows, gathering from all rows."""
        k = _vp()
        _call(load().s3dsp_kmap_build_subm3_rows, self.handle, hsh.handle, n_out, ctypes.byref(k))
        return Kmap(self, k.value, n_out)

    def kmap_subm3_range(self, hsh: Hash, row_begin: int, row_end: int) -> Kmap:
        """Submanifold map of hash rows [row_begin, row_end), gathering from all rows."""
        k = _vp()
        _call(load().s3dsp_kmap_build_subm3_range, self.handle, hsh.handle, row_begin, row_end, ctypes.byref(k))
        return Kmap(self, k.value, row_end - row_begin)

    def subdivide(self, parents: Hash, child_coords_out) -> Kmap:
        k = _vp()
        _call(load().s3dsp_subdivide, self.handle, parents.handle, ptr(child_coords_out), ctypes.byref(k))
        return Kmap(self, k.value, parents.n * 8)

    def kmap_export_dense(self, kmap: Kmap, sentinel_mode: int, out):
        _call(load().s3dsp_kmap_export_dense, self.handle, kmap.handle, sentinel_mode, ptr(out))

    def kmap_pairs(self, kmap: Kmap, pin, pout):
        offs = (ctypes.c_int64 * 28)()
        _call(load().s3dsp_kmap_pairs, self.handle, kmap.handle, ptr(pin), ptr(pout), pin.numel(), offs)
        return list(offs)

    def kmap_pairs_noalloc(self, kmap: Kmap, pin, pout):
        """Same as kmap_pairs, but the library allocates no device memory
        (its scratch is a static device array; maps of at most 2^21 rows)."""
        offs = (ctypes.c_int64 * 28)()
        _call(load().s3dsp_kmap_pairs_noalloc, self.handle, kmap.handle, ptr(pin), ptr(pout), pin.numel(), offs)
        return list(offs)

    # ---- weights ---------------------------------------------------------
    @staticmethod
    def packed_bytes(precision: int, kvol: int, cin: int, cout: int) -> int:
        return load().s3dsp_weights_packed_bytes(precision, kvol, cin, cout)

    def weights_pack(self, src, layout: int, kvol: int, cin: int, cout: int, precision: int, dst):
        on_host = 0 if src.is_cuda else 1
        _call(load().s3dsp_weights_pack, self.handle, ptr(src), dtype_code(src), on_host, layout, kvol, cin, cout,
              precision, ptr(dst))

    # ---- conv ------------------------------------------------------------
    def conv_kernel(self, n_out: int, kvol: int, cin: int, cout: int, precision: int, flags: int = 0,
                    in_shift: int = 0) -> str:
        """Name of the kernel s3dsp_conv launches for this shape."""
        name = load().s3dsp_conv_kernel_shift(self.handle, n_out, kvol, cin, cout, in_shift, precision, flags)
        return name.decode() if name else ""

    def conv(self, kmap: Kmap | None, kvol: int, precision: int, x, weight, bias, out, cout: int,
             in_shift: int = 0, residual=None, res_shift: int = 0, flags: int = 0, pro=None,
             gn_partials=None, gn_groups: int = 0, n_out: int | None = None):
        n_out = out.shape[0] if n_out is None else n_out
        sub, mul, add = pro if pro is not None else (None, None, None)
        _call(load().s3dsp_conv, self.handle, kmap.handle if kmap else None, kvol, precision, ptr(x),
              dtype_code(x), x.shape[0], x.shape[1], in_shift, ptr(weight), ptr(bias), ptr(residual),
              dtype_code(residual) if residual is not None else 0, res_shift, ptr(out), dtype_code(out), n_out,
              cout, flags, ptr(sub), ptr(mul), ptr(add), ptr(gn_partials), gn_groups)

    def conv_concat(self, kmap: Kmap | None, kvol: int, precision: int, xa, xb, weight, bias, out, cout: int,
                    in_shift: int = 0, residual=None, res_shift: int = 0, flags: int = 0, pro=None,
                    gn_partials=None, gn_groups: int = 0, n_out: int | None = None):
        """conv over the channel concat of xa [n_in, ca] and xb [n_in, cb] (never built)."""
        assert xa.dtype == xb.dtype and xa.shape[0] == xb.shape[0]
        n_out = out.shape[0] if n_out is None else n_out
        sub, mul, add = pro if pro is not None else (None, None, None)
        _call(load().s3dsp_conv_concat, self.handle, kmap.handle if kmap else None, kvol, precision, ptr(xa),
              xa.shape[1], ptr(xb), xb.shape[1], dtype_code(xa), xa.shape[0], in_shift, ptr(weight), ptr(bias),
              ptr(residual), dtype_code(residual) if residual is not None else 0, res_shift, ptr(out),
              dtype_code(out), n_out, cout, flags, ptr(sub), ptr(mul), ptr(add), ptr(gn_partials), gn_groups)

    def kmap_compose(self, kmap: Kmap, rows, n_rows_in: int) -> Kmap:
        """Map whose entries are rows[kmap entry] (rows: device int32 [kmap input rows])."""
        k = _vp()
        _call(load().s3dsp_kmap_compose, self.handle, kmap.handle, ptr(rows), n_rows_in, ctypes.byref(k))
        return Kmap(self, k.value, kmap.rows)

    # ---- norms -----------------------------------------------------------
    @staticmethod
    def gn_partials_count(n_rows: int, channels: int, groups: int) -> int:
        return load().s3dsp_gn_partials_count(n_rows, channels, groups)

    def gn_stats(self, x, groups: int, partials):
        _call(load().s3dsp_gn_stats, self.handle, ptr(x), dtype_code(x), x.shape[0], x.shape[1], groups,
              ptr(partials))

    def gn_finalize(self, partials, n_rows: int, c: int, groups: int, eps: float, gamma, beta, sub, mul, add):
        _call(load().s3dsp_gn_finalize, self.handle, ptr(partials), n_rows, c, groups, eps, ptr(gamma), ptr(beta),
              ptr(sub), ptr(mul), ptr(add))

    def channel_affine(self, x, sub, mul, add, silu: bool, y):
        _call(load().s3dsp_channel_affine, self.handle, ptr(x), dtype_code(x), x.shape[0], x.shape[1], ptr(sub),
              ptr(mul), ptr(add), int(silu), ptr(y), dtype_code(y))

    def layer_norm(self, x, eps: float, y, gamma=None, beta=None, mod_scale=None, mod_shift=None,
                   silu: bool = False):
        _call(load().s3dsp_layer_norm, self.handle, ptr(x), dtype_code(x), x.shape[0], x.shape[1], eps, ptr(gamma),
              ptr(beta), ptr(mod_scale), ptr(mod_shift), int(silu), ptr(y), dtype_code(y))

    def layer_norm_concat(self, xa, xb, eps: float, y, gamma=None, beta=None, mod_scale=None, mod_shift=None,
                          silu: bool = False):
        """LayerNorm over the channel concat of xa [n, ca] and xb [n, cb] into y [n, ca + cb]."""
        assert xa.dtype == xb.dtype and xa.shape[0] == xb.shape[0]
        _call(load().s3dsp_layer_norm_concat, self.handle, ptr(xa), xa.shape[1], ptr(xb), xb.shape[1], dtype_code(xa),
              xa.shape[0], eps, ptr(gamma), ptr(beta), ptr(mod_scale), ptr(mod_shift), int(silu), ptr(y),
              dtype_code(y))

    def convert(self, x, y):
        _call(load().s3dsp_convert, self.handle, ptr(x), dtype_code(x), ptr(y), dtype_code(y), x.numel())

    # ---- SLat coarse tables / down / up ----------------------------------
    def slat_tables(self, fine: Hash) -> SlatTables:
        t = _vp()
        _call(load().s3dsp_slat_tables_build, self.handle, fine.handle, ctypes.byref(t))
        return SlatTables(self, t.value, fine.n)

    def slat_tables_export(self, t: SlatTables, f2c=None, children=None, inv=None, coarse_coords=None):
        _call(load().s3dsp_slat_tables_export, self.handle, t.handle, ptr(f2c), ptr(children), ptr(inv),
              ptr(coarse_coords))

    def slat_downsample(self, t: SlatTables, x, y):
        _call(load().s3dsp_slat_downsample, self.handle, t.handle, ptr(x), dtype_code(x), x.shape[1], ptr(y),
              dtype_code(y))

    def slat_upsample(self, t: SlatTables, x, y):
        _call(load().s3dsp_slat_upsample, self.handle, t.handle, ptr(x), dtype_code(x), x.shape[1], ptr(y),
              dtype_code(y))

    # ---- block drivers ---------------------------------------------------
    def res_block_gn(self, kmap: Kmap, precision: int, x, w1, b1, gamma, beta, w2, b2, out, groups=32, eps=1e-5):
        _call(load().s3dsp_res_block_gn, self.handle, kmap.handle, precision, ptr(x), x.shape[0], x.shape[1],
              ptr(w1), ptr(b1), ptr(gamma), ptr(beta), ptr(w2), ptr(b2), groups, eps, ptr(out))

    def res_block_gn_host(self, precision: int, coords_h, x_h, w1, b1, gamma, beta, w2, b2, out_h, groups=32,
                          eps=1e-5):
        _call(load().s3dsp_res_block_gn_host, self.handle, precision, ptr(coords_h), coords_h.shape[0], ptr(x_h),
              x_h.shape[1], ptr(w1), ptr(b1), ptr(gamma), ptr(beta), ptr(w2), ptr(b2), groups, eps, ptr(out_h))

    def res_block_gn_host_queued(self, precision: int, coords_h, x_h, w1, b1, gamma, beta, w2, b2, out_h,
                                 groups=32, eps=1e-5):
        """Queued form of res_block_gn_host: returns once the work is on the
        context's stream (a DEFERRED_CHECKS context); out_h is ready when the
        stream gets there."""
        _call(load().s3dsp_res_block_gn_host_queued, self.handle, precision, ptr(coords_h), coords_h.shape[0],
              ptr(x_h), x_h.shape[1], ptr(w1), ptr(b1), ptr(gamma), ptr(beta), ptr(w2), ptr(b2), groups, eps,
              ptr(out_h))

    def mesh_upsample_level(self, parents: Hash, precision: int, x, cout, gn1_w, gn1_b, conv1_w, conv1_b, gn2_w,
                            gn2_b, conv2_w, conv2_b, skip_w, skip_b, child_coords, out):
        _call(load().s3dsp_mesh_upsample_level, self.handle, parents.handle, precision, ptr(x), x.shape[1], cout,
              ptr(gn1_w), ptr(gn1_b), ptr(conv1_w), ptr(conv1_b), ptr(gn2_w), ptr(gn2_b), ptr(conv2_w),
              ptr(conv2_b), ptr(skip_w), ptr(skip_b), ptr(child_coords), ptr(out))

    def mesh_upsample_level_host(self, precision: int, parent_coords_h, x_h, cout, gn1_w, gn1_b, conv1_w, conv1_b,
                                 gn2_w, gn2_b, conv2_w, conv2_b, skip_w, skip_b, child_coords_h, out_h):
        _call(load().s3dsp_mesh_upsample_level_host, self.handle, precision, ptr(parent_coords_h),
              parent_coords_h.shape[0], ptr(x_h), x_h.shape[1], cout, ptr(gn1_w), ptr(gn1_b), ptr(conv1_w),
              ptr(conv1_b), ptr(gn2_w), ptr(gn2_b), ptr(conv2_w), ptr(conv2_b), ptr(skip_w), ptr(skip_b),
              ptr(child_coords_h), ptr(out_h))

    def slat_res_block_concat(self, kmap: Kmap, precision: int, xa, xb, cout, norm1_w, norm1_b, conv1_w, conv1_b,
                              mod_scale, mod_shift, conv2_w, conv2_b, skip_w, skip_b, out, up_rows=None):
        """s3dsp_slat_res_block_concat: xb None for one source; up_rows (device
        int32 [kmap rows]) for a block on the nearest upsample of coarse xa/xb."""
        _call(load().s3dsp_slat_res_block_concat, self.handle, kmap.handle, ptr(up_rows), precision, ptr(xa),
              xa.shape[1], ptr(xb), 0 if xb is None else xb.shape[1], xa.shape[0], cout, ptr(norm1_w), ptr(norm1_b),
              ptr(conv1_w), ptr(conv1_b), ptr(mod_scale), ptr(mod_shift), ptr(conv2_w), ptr(conv2_b), ptr(skip_w),
              ptr(skip_b), ptr(out))

    def slat_res_block(self, kmap: Kmap, precision: int, x, cout, norm1_w, norm1_b, conv1_w, conv1_b, mod_scale,
                       mod_shift, conv2_w, conv2_b, skip_w, skip_b, out):
        _call(load().s3dsp_slat_res_block, self.handle, kmap.handle, precision, ptr(x), x.shape[0], x.shape[1], cout,
              ptr(norm1_w), ptr(norm1_b), ptr(conv1_w), ptr(conv1_b), ptr(mod_scale), ptr(mod_shift), ptr(conv2_w),
              ptr(conv2_b), ptr(skip_w), ptr(skip_b), ptr(out))
