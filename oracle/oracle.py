"""TEST INFRASTRUCTURE ONLY: ctypes front-end of the CPU oracle.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, as the checker or as the timed CPU comparator — never the product
path. Two libraries are reachable from here:

* ``libs3d_oracle.so`` — our restatement (oracle/s3d_oracle.cpp). Integer
  tables are pinned bit-exactly to the reference; the float ops restate the
  reference's GGML op order and are PARITY UNPINNED against GGML itself (the
  GGML submodule is absent), cross-checked against dense float64 torch ops.
* ``_ref/libsparse_ops_ref.so`` — the reference's own sparse_ops.cpp
  (SlatTables::build, MeshSubdivideTables::build) compiled unchanged, when it
  was built (it needs the reference tree at build time).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libs3d_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsparse_ops_ref.so")

_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_c_i64 = ctypes.c_int64
_c_i32 = ctypes.c_int32
_vp = ctypes.c_void_p

_lib = None
_ref = None


def build_oracle() -> str:
    """Compile the restatement (gcc only; works on any box with the image)."""
    subprocess.run(["make", "-s", "-C", HERE, "libs3d_oracle.so"], check=True)
    return ORACLE_SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO) or (
                os.path.getmtime(ORACLE_SO) < os.path.getmtime(os.path.join(HERE, "s3d_oracle.cpp"))):
            build_oracle()
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_slat_tables.restype = _c_i64
        L.oracle_slat_tables.argtypes = [_i32p, _c_i64, _i32p, _i32p, _f32p, _i32p, _i32p, _i32p]
        L.oracle_mesh_subdivide.restype = _c_i32
        L.oracle_mesh_subdivide.argtypes = [_i32p, _c_i64, _i32p, _i32p]
        L.oracle_subm_conv_slat.restype = None
        L.oracle_subm_conv_slat.argtypes = [_f32p, _c_i64, _c_i64, _i32p, _c_i64, _f32p, _vp,
                                            _c_i64, _f32p, _c_i32, _c_i32]
        L.oracle_subm_conv_mesh.restype = None
        L.oracle_subm_conv_mesh.argtypes = [_f32p, _c_i64, _c_i64, _vp, _c_i32, _c_i32, _c_i64,
                                            _f32p, _vp, _c_i64, _f32p, _c_i32, _c_i32]
        L.oracle_linear.restype = None
        L.oracle_linear.argtypes = [_f32p, _c_i64, _c_i64, _c_i32, _f32p, _vp, _c_i64, _f32p,
                                    _c_i32]
        L.oracle_group_norm.restype = None
        L.oracle_group_norm.argtypes = [_f32p, _c_i64, _c_i64, _c_i32, ctypes.c_float, _vp, _vp,
                                        _c_i32, _f32p]
        L.oracle_layer_norm.restype = None
        L.oracle_layer_norm.argtypes = [_f32p, _c_i64, _c_i64, ctypes.c_float, _vp, _vp, _vp, _vp,
                                        _c_i32, _f32p]
        L.oracle_downsample_mean.restype = None
        L.oracle_downsample_mean.argtypes = [_f32p, _c_i64, _c_i64, _i32p, _f32p, _c_i64, _f32p]
        L.oracle_upsample_nearest.restype = None
        L.oracle_upsample_nearest.argtypes = [_f32p, _c_i64, _c_i64, _i32p, _c_i64, _f32p]
        L.oracle_occupancy_coords.restype = _c_i64
        L.oracle_occupancy_coords.argtypes = [_f32p, _c_i32, _c_i32, _c_i32, _c_i32, _i32p]
        L.oracle_prune_surface.restype = _c_i64
        L.oracle_prune_surface.argtypes = [_i32p, _c_i64, _c_i32, _i32p]
        L.oracle_downsample_coords.restype = _c_i64
        L.oracle_downsample_coords.argtypes = [_i32p, _c_i64, _c_i64, _c_i32, ctypes.c_uint32, _i32p]
        L.oracle_gs_window_tables.restype = _c_i64
        L.oracle_gs_window_tables.argtypes = [_i32p, _c_i64, _c_i32, _c_i32, _i32p, _i32p, _i32p]
        L.oracle_ape.restype = None
        L.oracle_ape.argtypes = [_i32p, _c_i64, _c_i32, _f32p]
        L.oracle_flexicubes.restype = _c_i32
        L.oracle_flexicubes.argtypes = [_f32p, _i32p, _c_i64, _vp, _vp, _vp, _vp]
        L.oracle_flexicubes_fetch.restype = None
        L.oracle_flexicubes_fetch.argtypes = [_vp] * 6
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError("reference table builder not built: " + REF_SO)
        L = ctypes.CDLL(REF_SO)
        L.ref_slat_tables.restype = _c_i64
        L.ref_slat_tables.argtypes = [_i32p, _c_i64, _c_i32, _i32p, _i32p, _f32p, _i32p, _i32p]
        L.ref_mesh_subdivide.restype = _c_i32
        L.ref_mesh_subdivide.argtypes = [_i32p, _c_i64, _i32p, _i32p]
        L.ref_gs_tables.restype = _c_i64
        L.ref_gs_tables.argtypes = [_i32p, _c_i64, _c_i32, _i32p, _i32p, _i32p, _vp]
        L.ref_flexicubes_tables.restype = None
        L.ref_flexicubes_tables.argtypes = [_vp, _vp, _vp]
        L.ref_flexicubes.restype = _c_i32
        L.ref_flexicubes.argtypes = [_f32p, _i32p, _c_i64, _vp, ctypes.c_char_p, _c_i64]
        L.ref_flexicubes_fetch.restype = None
        L.ref_flexicubes_fetch.argtypes = [_vp] * 6
        _ref = L
    return _ref


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ---------------------------------------------------------------------------
# integer tables
# ---------------------------------------------------------------------------
def slat_tables(coords: np.ndarray, use_ref: bool = False) -> dict | None:
    """SlatTables (sparse_ops.cpp:49-173). Returns None when the builder fails."""
    coords = _c(coords, np.int32).reshape(-1, 4)
    nf = len(coords)
    f2c = np.zeros(max(nf, 1), np.int32)
    ch = np.zeros(max(8 * nf, 1), np.int32)
    inv = np.zeros(max(nf, 1), np.float32)
    cf = np.zeros(max(27 * nf, 1), np.int32)
    cc = np.zeros(max(27 * nf, 1), np.int32)
    if use_ref:
        nc = ref_lib().ref_slat_tables(coords.reshape(-1) if nf else np.zeros(4, np.int32), nf, 6,
                                       f2c, ch, inv, cf, cc)
        ccoords = None
    else:
        ccoords = np.zeros(max(4 * nf, 1), np.int32)
        nc = lib().oracle_slat_tables(coords.reshape(-1) if nf else np.zeros(4, np.int32), nf,
                                      f2c, ch, inv, cf, cc, ccoords)
    if nc < 0:
        return None
    out = dict(nf=nf, nc=int(nc), fine_to_coarse=f2c[:nf], coarse_children=ch[:8 * nc],
               coarse_inv_count=inv[:nc], conv_fine=cf[:27 * nf], conv_coarse=cc[:27 * nc])
    if ccoords is not None:
        out["coarse_coords"] = ccoords[:4 * nc].reshape(nc, 4)
    return out


def mesh_subdivide(parents: np.ndarray, use_ref: bool = False):
    """MeshSubdivideTables (sparse_ops.cpp:272-404) -> (child_coords [8N,4],
    neighbors [8N,27]) or None when the builder rejects the input."""
    parents = _c(parents, np.int32).reshape(-1, 4)
    n = len(parents)
    cc = np.zeros(max(32 * n, 4), np.int32)
    nb = np.zeros(max(8 * 27 * n, 1), np.int32)
    src = parents.reshape(-1) if n else np.zeros(4, np.int32)
    ok = (ref_lib().ref_mesh_subdivide if use_ref else lib().oracle_mesh_subdivide)(src, n, cc, nb)
    if not ok:
        return None
    return cc[:32 * n].reshape(8 * n, 4), nb[:8 * 27 * n].reshape(8 * n, 27)


def gs_window_tables(coords: np.ndarray, shift_index: int, use_ref: bool = False):
    """GsTables::build (sparse_ops.cpp:182-270), shift (0,0,0) or (4,4,4):
    (bkt_idx [n], bwd_idx [n], buckets [k, 3] = {len, off, n_win})."""
    coords = _c(coords, np.int32).reshape(-1, 4)
    n = len(coords)
    bkt = np.zeros(max(n, 1), np.int32)
    bwd = np.zeros(max(n, 1), np.int32)
    bk = np.zeros((max(n, 1), 3), np.int32)
    if use_ref:
        k = ref_lib().ref_gs_tables(coords.reshape(-1), n, shift_index, bkt, bwd, bk.reshape(-1), None)
    else:
        k = lib().oracle_gs_window_tables(coords.reshape(-1), n, 4 * shift_index, 8, bkt, bwd, bk.reshape(-1))
    if k < 0:
        return None
    return bkt[:n], bwd[:n], bk[:k]


def ape(coords: np.ndarray, channels: int = 768, use_ref: bool = False) -> np.ndarray:
    """AbsolutePositionEmbedder of GsTables::build: [n, channels] f32."""
    coords = _c(coords, np.int32).reshape(-1, 4)
    n = len(coords)
    out = np.zeros((n, channels), np.float32)
    if use_ref:
        assert channels == 768
        d = np.zeros(max(n, 1), np.int32)
        b = np.zeros((max(n, 1), 3), np.int32)
        ref_lib().ref_gs_tables(coords.reshape(-1), n, 0, d, d.copy(), b.reshape(-1),
                                out.ctypes.data_as(ctypes.c_void_p))
    else:
        lib().oracle_ape(coords.reshape(-1), n, channels, out.reshape(-1))
    return out


def occupancy_coords(occ: np.ndarray, batch: int = 0) -> np.ndarray:
    """SS occupancy argwhere (session.cpp:1436-1441): occ [X, Y, Z] > 0 ->
    int32 rows (batch, x, y, z), x-major."""
    occ = _c(occ, np.float32)
    nx, ny, nz = occ.shape
    out = np.zeros((max(occ.size, 1), 4), np.int32)
    n = lib().oracle_occupancy_coords(occ.reshape(-1), nx, ny, nz, batch, out.reshape(-1))
    return out[:n]


def prune_surface(coords: np.ndarray, dist: int = 1) -> np.ndarray:
    """prune_surface_coords (session.cpp:129-166)."""
    coords = _c(coords, np.int32).reshape(-1, 4)
    out = np.zeros((max(len(coords), 1), 4), np.int32)
    n = lib().oracle_prune_surface(coords.reshape(-1) if len(coords) else out.reshape(-1), len(coords), dist,
                                   out.reshape(-1))
    return out[:n]


def downsample_coords(coords: np.ndarray, max_coords: int = 42000, factor: int = 2, seed: int = 42) -> np.ndarray:
    """downsample_coords (session.cpp:168-236)."""
    coords = _c(coords, np.int32).reshape(-1, 4)
    out = np.zeros((max(len(coords), 1), 4), np.int32)
    n = lib().oracle_downsample_coords(coords.reshape(-1) if len(coords) else out.reshape(-1), len(coords),
                                       max_coords, factor, seed, out.reshape(-1))
    return out[:n]


# ---------------------------------------------------------------------------
# float ops (GGML order restatement; see module docstring)
# ---------------------------------------------------------------------------
def subm_conv_slat(feat, nbr, w_slat, bias, accum64=False, threads=0):
    """SLat SubMConv3d: feat [n_in, Cin], nbr [n_out, 27] (entries outside
    [0, n_in) read zeros), w_slat [Cout, 27*Cin] -> [n_out, Cout]."""
    feat = _c(feat, np.float32)
    n_in, cin = feat.shape
    nbr = _c(nbr, np.int32).reshape(-1, 27)
    cout = w_slat.shape[0]
    out = np.empty((len(nbr), cout), np.float32)
    lib().oracle_subm_conv_slat(feat.reshape(-1), n_in, cin, nbr.reshape(-1), len(nbr),
                                _c(w_slat, np.float32).reshape(-1),
                                _ptr(_c(bias, np.float32) if bias is not None else None), cout,
                                out.reshape(-1), int(accum64), threads)
    return out


def subm_conv_mesh(feat, nbr, w_packed, bias, cout, kvol=27, gather_shift=0, n_out=None,
                   accum64=False, threads=0):
    """mesh SubMConv3d: per-offset GEMMs summed o=0..kvol-1, then bias.
    w_packed [kvol, Cout*Cin]; nbr [n_out, 27] with -1 = missing (ignored for
    kvol == 1); gathered rows are (src >> gather_shift)."""
    feat = _c(feat, np.float32)
    n_in, cin = feat.shape
    if kvol == 1:
        nbr_arr = None
        assert n_out is not None
    else:
        nbr_arr = _c(nbr, np.int32).reshape(-1, 27)
        n_out = len(nbr_arr)
    out = np.empty((n_out, cout), np.float32)
    keep = bias if bias is None else _c(bias, np.float32)
    lib().oracle_subm_conv_mesh(feat.reshape(-1), n_in, cin, _ptr(nbr_arr), kvol, gather_shift,
                                n_out, _c(w_packed, np.float32).reshape(-1), _ptr(keep), cout,
                                out.reshape(-1), int(accum64), threads)
    return out


def linear(x, w, bias, row_shift=0, n_out=None, threads=0):
    """gb_linear: x [n_in, Cin] @ W[Cout, Cin]^T + b; row r reads x[r >> row_shift]."""
    x = _c(x, np.float32)
    cin = x.shape[1]
    cout = w.shape[0]
    n_out = len(x) << row_shift if n_out is None else n_out
    out = np.empty((n_out, cout), np.float32)
    keep = bias if bias is None else _c(bias, np.float32)
    lib().oracle_linear(x.reshape(-1), n_out, cin, row_shift, _c(w, np.float32).reshape(-1),
                        _ptr(keep), cout, out.reshape(-1), threads)
    return out


def group_norm(x, groups, eps=1e-5, gamma=None, beta=None, silu=False):
    x = _c(x, np.float32)
    n, c = x.shape
    out = np.empty_like(x)
    g = None if gamma is None else _c(gamma, np.float32)
    b = None if beta is None else _c(beta, np.float32)
    lib().oracle_group_norm(x.reshape(-1), n, c, groups, eps, _ptr(g), _ptr(b), int(silu),
                            out.reshape(-1))
    return out


def layer_norm(x, eps=1e-6, gamma=None, beta=None, mod_scale=None, mod_shift=None, silu=False):
    x = _c(x, np.float32)
    n, c = x.shape
    out = np.empty_like(x)
    keep = [None if a is None else _c(a, np.float32) for a in (gamma, beta, mod_scale, mod_shift)]
    lib().oracle_layer_norm(x.reshape(-1), n, c, eps, *[_ptr(a) for a in keep], int(silu),
                            out.reshape(-1))
    return out


def silu(x):
    x = np.asarray(x, np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def downsample_mean(x, children, inv_count):
    x = _c(x, np.float32)
    nf, ch = x.shape
    nc = len(inv_count)
    out = np.empty((nc, ch), np.float32)
    lib().oracle_downsample_mean(x.reshape(-1), nf, ch, _c(children, np.int32).reshape(-1),
                                 _c(inv_count, np.float32), nc, out.reshape(-1))
    return out


def upsample_nearest(x, f2c):
    x = _c(x, np.float32)
    nc, ch = x.shape
    f2c = _c(f2c, np.int32)
    out = np.empty((len(f2c), ch), np.float32)
    lib().oracle_upsample_nearest(x.reshape(-1), nc, ch, f2c, len(f2c), out.reshape(-1))
    return out


# ---------------------------------------------------------------------------
# composite blocks (op sequences of the reference graphs)
# ---------------------------------------------------------------------------
def resblock_gn(feats, nbr_slat, w1, b1, gamma, beta, w2, b2, groups=32, eps=1e-5, threads=0):
    """Config 2 residual block: conv3 -> GroupNorm(32) -> SiLU -> conv3 -> + x.
    GroupNorm/SiLU follow mesh_decoder_graph.cpp:16-30/:117-121, the convs the
    SLat single-GEMM form (slat_flow_graph.cpp:112-155)."""
    h = subm_conv_slat(feats, nbr_slat, w1, b1, threads=threads)
    h = group_norm(h, groups, eps, gamma, beta, silu=True)
    h = subm_conv_slat(h, nbr_slat, w2, b2, threads=threads)
    return h + feats


def mesh_upsample_level(x, neighbors, p, threads=0, taps=None):
    """MeshUpsampleGraph::build (mesh_decoder_graph.cpp:42-132) for one level.
    x [Np, Cin] parent features, neighbors [8Np, 27] child table (-1 missing),
    p: dict of gn1_w, gn1_b, conv1_w (packed [27, Cout*Cin]), conv1_b, gn2_w,
    gn2_b, conv2_w, conv2_b, skip_w ([1, Cout*Cin] packed 1x1), skip_b."""
    cin = x.shape[1]
    cout = len(p["conv1_b"])
    n_child = len(neighbors)
    h = group_norm(x, 32, 1e-5, p["gn1_w"], p["gn1_b"], silu=True)          # norm1, silu1
    h = subm_conv_mesh(h, neighbors, p["conv1_w"], p["conv1_b"], cout, 27, 3, threads=threads)
    if taps is not None:
        taps["conv1"] = h
    h = group_norm(h, 32, 1e-5, p["gn2_w"], p["gn2_b"], silu=True)          # norm2, silu2
    h = subm_conv_mesh(h, neighbors, p["conv2_w"], p["conv2_b"], cout, 27, 0, threads=threads)
    if taps is not None:
        taps["conv2"] = h
    skip = subm_conv_mesh(x, None, p["skip_w"], p["skip_b"], cout, 1, 3, n_out=n_child,
                          threads=threads)
    if taps is not None:
        taps["skip"] = skip
    return h + skip


def slat_res_block(x, nbr_slat, norm1_w, norm1_b, w1, b1, mod_scale, mod_shift, w2, b2, skip_w=None, skip_b=None,
                   threads=0, accum64=False):
    """res_block of slat_flow_graph.cpp:216-275 (no down/up): LayerNorm(1e-6,
    affine) -> SiLU -> conv1 -> LayerNorm(1e-6) -> modulate -> SiLU -> conv2
    -> + skip (identity, or Linear when the width changes, :266-272).
    accum64: the convs' dot products in float64 (a second check)."""
    h = layer_norm(x, 1e-6, norm1_w, norm1_b, silu=True)
    h = subm_conv_slat(h, nbr_slat, w1, b1, accum64=accum64, threads=threads)
    h = layer_norm(h, 1e-6, None, None, mod_scale, mod_shift, silu=True)
    h = subm_conv_slat(h, nbr_slat, w2, b2, accum64=accum64, threads=threads)
    skip = x if skip_w is None else linear(x, skip_w, skip_b, threads=threads)
    return h + skip


def slat_sparse_forward(coords, x, p, mods, mid=None, threads=0, accum64=False, taps=None):
    """The SLat flow generator's sparse stages, in the reference's op order
    (slat_flow_graph.cpp): input_layer Linear (:283-285); input_blocks.0
    res_block on the fine map (:290-291); 2x mean-pool down (:159-183) +
    input_blocks.1 res_block on the coarse map with a Linear skip (:294-296);
    `mid` (the dense APE + transformer torso, :298-460; identity when None);
    out_blocks.0: ggml_concat(h, skip1) -> nearest upsample (:185-190) ->
    res_block with a Linear skip (:463-495); out_blocks.1: ggml_concat(h,
    skip0) -> res_block with a Linear skip (:496-524); LayerNorm(1e-6, no
    affine) -> out_layer Linear (:527-531). Tables by SlatTables::build
    (sparse_ops.cpp:49-173). p / mods as sam3d.cpp_b200/slat.py makes them.
    Returns [nf, out_ch] f32; `taps` (a dict) receives the intermediates."""
    t = slat_tables(coords)
    nf = len(coords)
    nc = len(t["coarse_inv_count"])
    fine = t["conv_fine"].reshape(nf, 27)
    coarse = t["conv_coarse"].reshape(nc, 27)

    def block(name, xin, nbr):
        b = p[name]
        sc, sh = mods[name]
        return slat_res_block(xin, nbr, b["norm1_w"], b["norm1_b"], b["conv1_w"], b["conv1_b"], sc, sh, b["conv2_w"],
                              b["conv2_b"], b.get("skip_w"), b.get("skip_b"), threads=threads, accum64=accum64)

    h = linear(x, p["input_layer"]["w"], p["input_layer"]["b"], threads=threads)
    skip0 = block("input_blocks.0", h, fine)
    d = downsample_mean(skip0, t["coarse_children"], t["coarse_inv_count"])
    skip1 = block("input_blocks.1", d, coarse)
    h = skip1 if mid is None else mid(skip1)
    xin = upsample_nearest(np.concatenate([h, skip1], axis=1), t["fine_to_coarse"])
    h = block("out_blocks.0", xin, fine)
    ob0 = h
    xin = np.concatenate([h, skip0], axis=1)
    h = block("out_blocks.1", xin, fine)
    ob1 = h
    h = layer_norm(h, 1e-6)
    out = linear(h, p["out_layer"]["w"], p["out_layer"]["b"], threads=threads)
    if taps is not None:
        taps.update(skip0=skip0, skip1=skip1, out_blocks0=ob0, out_blocks1=ob1, out=out)
    return out


# ---------------------------------------------------------------------------
# FlexiCubes extraction (src/objects_runtime/mesh_extractor.cpp:95-377)
# ---------------------------------------------------------------------------
FLEXICUBES_ERRORS = {-1: "invalid mesh decoder tensor", -2: "mesh extraction currently requires batch one",
                     -3: "mesh cube coordinate outside resolution 256", -4: "duplicate mesh cube coordinate"}


def ref_flexicubes_tables():
    """The reference's DMC tables, read from its compiled extractor:
    dict(dmc int8 [256, 4, 7], num_dual int8 [256], check int16 [256, 5])."""
    dmc = np.zeros((256, 4, 7), np.int8)
    nd = np.zeros(256, np.int8)
    ck = np.zeros((256, 5), np.int16)
    ref_lib().ref_flexicubes_tables(_ptr(dmc), _ptr(nd), _ptr(ck))
    return dict(dmc=dmc, num_dual=nd, check=ck)


def flexicubes(raw: np.ndarray, coords: np.ndarray, tables=None, use_ref: bool = False):
    """extract_object_mesh with taps: dict(vertices [D, 3], attrs [D, 6],
    faces [F, 3], surface [S] dense cube ids, cases [S], edges [E, 2]); raises
    ValueError with the reference's message on its input errors. `tables`
    (dmc, num_dual, check) is needed by the restatement only."""
    raw = _c(raw, np.float32).reshape(-1, 101)
    coords = _c(coords, np.int32).reshape(-1, 4)
    n = len(coords)
    counts = np.zeros(4, np.int64)
    if use_ref:
        err = ctypes.create_string_buffer(256)
        rc = ref_lib().ref_flexicubes(raw.reshape(-1), coords.reshape(-1), n, _ptr(counts), err, 256)
        if rc != 0:
            raise ValueError(err.value.decode())
        fetch = ref_lib().ref_flexicubes_fetch
    else:
        dmc = _c(tables["dmc"], np.int8)
        nd = _c(tables["num_dual"], np.int8)
        ck = _c(tables["check"], np.int16)
        rc = lib().oracle_flexicubes(raw.reshape(-1), coords.reshape(-1), n, _ptr(dmc), _ptr(nd), _ptr(ck),
                                     _ptr(counts))
        if rc != 0:
            raise ValueError(FLEXICUBES_ERRORS[rc])
        fetch = lib().oracle_flexicubes_fetch
    d, f, ns, ne = (int(v) for v in counts)
    out = dict(vertices=np.zeros((d, 3), np.float32), attrs=np.zeros((d, 6), np.float32),
               faces=np.zeros((f, 3), np.int32), surface=np.zeros(ns, np.int32), cases=np.zeros(ns, np.int32),
               edges=np.zeros((ne, 2), np.int32))
    fetch(*(_ptr(out[k]) for k in ("vertices", "attrs", "faces", "surface", "cases", "edges")))
    return out


# ---------------------------------------------------------------------------
# GS decoder Swin torso (src/objects_runtime/gs_decoder_graph.cpp:13-155)
# ---------------------------------------------------------------------------
def _norm64(x, eps):
    """ggml_norm: (x - mean) / sqrt(var + eps), biased variance, no affine."""
    m = x.mean(axis=1, keepdims=True)
    d = x - m
    return d / np.sqrt((d * d).mean(axis=1, keepdims=True) + eps)


def _gelu64(x):
    """GELU, tanh form (the approximation ggml_gelu evaluates; GGML's CPU
    path reads it from an f16 table, which this float64 restatement does not)."""
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def window_attention(qkv, heads, buckets, bkt_idx):
    """The bucket loop of gs_decoder_graph.cpp:88-121 in float64: qkv [n, 3c]
    rows in bucket order; per bucket {len, off, n_win} and per head,
    softmax(q k^T / sqrt(d)) v within each window of `len` consecutive rows;
    the result back in token order (row i -> token bkt_idx[i])."""
    qkv = np.asarray(qkv, np.float64)
    n, c3 = qkv.shape
    c = c3 // 3
    d = c // heads
    acc = np.zeros((n, c), np.float64)
    for len_, off, nw in buckets:
        blk = qkv[off:off + len_ * nw].reshape(nw, len_, 3, heads, d)
        q, k, v = blk[:, :, 0], blk[:, :, 1], blk[:, :, 2]          # [nw, len, H, d]
        s = np.einsum("wqhd,wkhd->whqk", q, k) / np.sqrt(d)
        s = np.exp(s - s.max(axis=-1, keepdims=True))
        s /= s.sum(axis=-1, keepdims=True)
        o = np.einsum("whqk,wkhd->wqhd", s, v)
        acc[off:off + len_ * nw] = o.reshape(len_ * nw, c)
    out = np.zeros_like(acc)
    out[np.asarray(bkt_idx)] = acc
    return out


def gs_torso_forward(coords, x, p, taps=None):
    """The GS decoder in the reference's op order, float64: input Linear +
    APE (:37-48); per block (tables of shift 0 for even blocks, (4,4,4) for
    odd): norm(1e-6) -> bucket-order gather -> q, k, v Linears -> window
    attention -> token order -> to_out Linear -> + h; norm(1e-6) -> Linear ->
    GELU -> Linear -> + h (:55-142); final norm(1e-5) -> out Linear
    (:146-151). Tables and APE by the restated GsTables::build. p as
    sam3d.cpp_b200/gs.py makes it."""
    heads = 12
    tabs = [gs_window_tables(coords, si) for si in (0, 1)]
    h = np.asarray(x, np.float64) @ np.asarray(p["input_layer"]["w"], np.float64).T + p["input_layer"]["b"]
    h = h + ape(coords, h.shape[1]).astype(np.float64)
    for i, b in enumerate(p["blocks"]):
        bkt, _, buckets = tabs[i % 2]
        hb = _norm64(h, 1e-6)[bkt]
        qkv = hb @ np.asarray(b["qkv"]["w"], np.float64).T + b["qkv"]["b"]
        ao = window_attention(qkv, heads, buckets, bkt)
        h = h + ao @ np.asarray(b["out"]["w"], np.float64).T + b["out"]["b"]
        g = _gelu64(_norm64(h, 1e-6) @ np.asarray(b["mlp0"]["w"], np.float64).T + b["mlp0"]["b"])
        h = h + g @ np.asarray(b["mlp2"]["w"], np.float64).T + b["mlp2"]["b"]
        if taps is not None:
            taps[f"block{i}"] = h
    return _norm64(h, 1e-5) @ np.asarray(p["out_layer"]["w"], np.float64).T + p["out_layer"]["b"]
