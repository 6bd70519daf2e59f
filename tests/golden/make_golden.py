"""Generates the committed golden fixtures of the sparse-table path.

Run in a container that has the reference tree (it is not needed afterwards):

    make -C oracle ref && python tests/golden/make_golden.py [REFERENCE_ROOT]

Every expected table here comes from the REFERENCE's own table builders
(SlatTables::build, MeshSubdivideTables::build in
src/objects_runtime/sparse_ops.cpp, compiled unchanged into
oracle/_ref/libsparse_ops_ref.so), never from our restatement. Outputs:

* kat_block3.npz   - the 3x3x3 voxel block at x,y,z in {30,31,32} used by the
                     reference's mesh capture (scripts/objects/
                     capture_mesh_reference.py:135-145), full tables;
* shell16.npz      - a small ellipsoid shell (res 16), full tables;
* edge_cases.npz   - multi-batch, negative coordinates and duplicated rows
                     (SlatTables) plus the reference's accept/reject verdicts
                     for MeshSubdivideTables;
* ss_occ_mask.npz  - occupancy bitmask (occ > 0) of the reference fixture
                     tests/objects_runtime/fixtures/ss_occ_f32.samt (a real 64^3
                     SS-decoder output), packed with np.packbits;
* digests.json     - sha256 of the reference tables for the larger sets
                     (config-1 shell, its subdivide, the pruned ss_occ set)
                     and of the reference's FlexiCubes topology for the
                     full-size extraction inputs;
* flexicubes_tables.npz - the DMC tables (dmc, num_dual, check) read out of
                     the reference's compiled extractor
                     (src/objects_runtime/flexicubes_tables.hpp, used by
                     mesh_extractor.cpp); the device extractor takes them as
                     an input;
* flexicubes_small.npz - extract_object_mesh output (with taps) for
                     workloads.flexicubes_input(8, 0), the input regenerated
                     from its seed.

`python tests/golden/make_golden.py --flexicubes` regenerates only the
FlexiCubes fixtures (and their digests entries).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "sam3d.cpp_b200"))
import oracle  # noqa: E402
import workloads  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).astype("<i4").tobytes()).hexdigest()


def sha_f(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).astype("<f4").tobytes()).hexdigest()


def ref_tables(coords):
    t = oracle.slat_tables(coords, use_ref=True)
    m = oracle.mesh_subdivide(coords, use_ref=True)
    return t, m


def block3():
    xyz = np.stack(np.meshgrid(np.arange(30, 33), np.arange(30, 33), np.arange(30, 33), indexing="ij"),
                   axis=-1).reshape(-1, 3)
    return np.concatenate([np.zeros((27, 1), np.int32), xyz.astype(np.int32)], axis=1)


def save_full(name, coords):
    t, m = ref_tables(coords)
    np.savez_compressed(os.path.join(HERE, name), coords=coords, nc=t["nc"],
                        fine_to_coarse=t["fine_to_coarse"], coarse_children=t["coarse_children"],
                        coarse_inv_count=t["coarse_inv_count"], conv_fine=t["conv_fine"],
                        conv_coarse=t["conv_coarse"], child_coords=m[0], neighbors=m[1])


def read_samt(path):
    with open(path, "rb") as f:
        magic, nd = struct.unpack("<Ii", f.read(8))
        assert magic == 0x544D4153, "not a SAMT file"
        ne = struct.unpack("<%dq" % nd, f.read(8 * nd))
        (typ,) = struct.unpack("<i", f.read(4))
        data = np.frombuffer(f.read(), dtype="<f4")
    assert typ == 0
    return ne, data


def occ_coords(mask3):
    """occ > 0 cells in (x, y, z) lexicographic order (session.cpp:1436-1441)."""
    x, y, z = np.nonzero(mask3)
    return np.stack([np.zeros_like(x), x, y, z], axis=1).astype(np.int32)


def prune_surface(coords):
    """prune_surface_coords (session.cpp:133-166): keep a voxel when any of its
    27 neighbours (itself included, grid exterior counting as empty) is empty;
    input order preserved."""
    occ = np.zeros((66, 66, 66), bool)
    occ[coords[:, 1] + 1, coords[:, 2] + 1, coords[:, 3] + 1] = True
    keep = np.zeros(len(coords), bool)
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                keep |= ~occ[coords[:, 1] + 1 + dx, coords[:, 2] + 1 + dy, coords[:, 3] + 1 + dz]
    return coords[keep]


FLEXICUBES_DIGEST_CASES = {"flexicubes_full64": dict(parent_res=64, seed=0),
                           "flexicubes_noisy16": dict(parent_res=16, seed=1, sdf_noise=3.0)}


def make_flexicubes():
    t = oracle.ref_flexicubes_tables()
    np.savez_compressed(os.path.join(HERE, "flexicubes_tables.npz"), **t)
    c, r = workloads.flexicubes_input(8, 0)
    m = oracle.flexicubes(r, c, use_ref=True)
    np.savez_compressed(os.path.join(HERE, "flexicubes_small.npz"), parent_res=8, seed=0, n=len(c), **m)
    out = {}
    for name, kw in FLEXICUBES_DIGEST_CASES.items():
        c, r = workloads.flexicubes_input(**kw)
        m = oracle.flexicubes(r, c, use_ref=True)
        out[name] = dict(kw, n=len(c), **{k: sha(m[k]) for k in ("faces", "surface", "cases", "edges")},
                         **{"n_" + k: len(m[k]) for k in ("vertices", "faces", "surface", "edges")})
    return out


def main():
    if not oracle.ref_available():
        raise SystemExit("build oracle/_ref first: make -C oracle ref")
    if "--flexicubes" in sys.argv[1:]:
        path = os.path.join(HERE, "digests.json")
        with open(path) as f:
            digests = json.load(f)
        digests.update(make_flexicubes())
        with open(path, "w") as f:
            json.dump(digests, f, indent=1, sort_keys=True)
        return
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("S3D_REFERENCE_ROOT", "")

    save_full("kat_block3.npz", block3())
    save_full("shell16.npz", workloads.ellipsoid_shell(16, seed=3))

    # edge cases
    rng = np.random.default_rng(7)
    multi = np.concatenate([
        np.concatenate([np.full((40, 1), b, np.int32), rng.integers(-3, 4, size=(40, 3)).astype(np.int32)], 1)
        for b in (0, 1, 2)])
    _, first = np.unique(multi, axis=0, return_index=True)
    multi_unique = multi[np.sort(first)]
    dup_rows = np.concatenate([multi_unique, multi_unique[[0, 5, 9]]], axis=0)
    edge = {}
    for name, c in (("multi", multi), ("multi_unique", multi_unique), ("dup_rows", dup_rows)):
        t = oracle.slat_tables(c, use_ref=True)
        m = oracle.mesh_subdivide(c, use_ref=True)
        edge[name + "_coords"] = c
        for k in ("fine_to_coarse", "coarse_children", "coarse_inv_count", "conv_fine", "conv_coarse"):
            edge[f"{name}_{k}"] = t[k]
        edge[name + "_nc"] = t["nc"]
        edge[name + "_mesh_ok"] = m is not None
        if m is not None:
            edge[name + "_child_coords"], edge[name + "_neighbors"] = m
    np.savez_compressed(os.path.join(HERE, "edge_cases.npz"), **edge)

    digests = {}
    shell = workloads.ellipsoid_shell(64, 0)
    t, m = ref_tables(shell)
    digests["config1_shell"] = dict(n=len(shell), coords=sha(shell), nc=t["nc"], conv_fine=sha(t["conv_fine"]),
                                    conv_coarse=sha(t["conv_coarse"]), fine_to_coarse=sha(t["fine_to_coarse"]),
                                    coarse_children=sha(t["coarse_children"]),
                                    coarse_inv_count=sha_f(t["coarse_inv_count"]),
                                    child_coords=sha(m[0]), neighbors=sha(m[1]))
    # second level of the mesh decoder: subdivide the children again
    m2 = oracle.mesh_subdivide(m[0], use_ref=True)
    digests["config1_subdivide2"] = dict(n=len(m[0]), child_coords=sha(m2[0]), neighbors=sha(m2[1]))

    if ref_root:
        samt = os.path.join(ref_root, "tests/objects_runtime/fixtures/ss_occ_f32.samt")
        ne, data = read_samt(samt)
        assert tuple(ne) == (64, 64, 64)
        mask = (data.reshape(64, 64, 64) > 0)  # flat = (x*64 + y)*64 + z
        np.savez_compressed(os.path.join(HERE, "ss_occ_mask.npz"), bits=np.packbits(mask.reshape(-1)))
        occ = occ_coords(mask)
        pruned = prune_surface(occ)
        t, m = ref_tables(pruned)
        digests["ss_occ_pruned"] = dict(n_occupied=len(occ), n=len(pruned), coords=sha(pruned), nc=t["nc"],
                                        conv_fine=sha(t["conv_fine"]), conv_coarse=sha(t["conv_coarse"]),
                                        fine_to_coarse=sha(t["fine_to_coarse"]),
                                        coarse_children=sha(t["coarse_children"]),
                                        coarse_inv_count=sha_f(t["coarse_inv_count"]),
                                        child_coords=sha(m[0]), neighbors=sha(m[1]))
    digests.update(make_flexicubes())
    with open(os.path.join(HERE, "digests.json"), "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)
    print(json.dumps({k: v.get("n") for k, v in digests.items()}))


if __name__ == "__main__":
    main()
