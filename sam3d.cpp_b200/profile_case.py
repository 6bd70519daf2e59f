"""Small, self-contained invocations of single kernels, for ncu captures.

  python sam3d.cpp_b200/profile_case.py conv2      # config-2 conv (C=256, 15,159 voxels), 128-row kernel
  python sam3d.cpp_b200/profile_case.py conv_sk    # 256^3 shell (241,978 voxels), C=256, stream-K kernel
  python sam3d.cpp_b200/profile_case.py tables     # hash + submanifold kmap of the 2.58M-voxel 512^3 shell
  python sam3d.cpp_b200/profile_case.py flexicubes # FlexiCubes extraction of 970,176 cubes at 256^3
  python sam3d.cpp_b200/profile_case.py conv1_tf32 # config-1 subm conv (C=64, 15,159 voxels) in 3xTF32
  python sam3d.cpp_b200/profile_case.py coords     # SS occupancy -> coords -> surface prune -> downsample (64^3 fixture)
  python sam3d.cpp_b200/profile_case.py gs_tables  # GS window tables (both shifts) + APE, config-2 coordinates

Each case warms up once, then runs the kernel(s) under test `--reps` times on
one stream, synchronising at the end; the process exits 0 on success. The
inputs are larger than L2 where the case allows it (conv_sk: 124 MB of bf16
features; tables: 41 MB of coordinates, 168 MB of table, 279 MB of map;
flexicubes: 392 MB of raw features, about 0.9 GB of dense grids and slots).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["conv2", "conv_sk", "tables", "flexicubes", "coords", "gs_tables", "conv1_tf32"])
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    import torch
    import s3dsp
    import workloads

    ctx = s3dsp.Context(0)
    P = s3dsp.PREC_BF16
    if a.case in ("conv2", "conv_sk"):
        coords = workloads.ellipsoid_shell(64 if a.case == "conv2" else 256, 0)
        n, c = len(coords), 256
        h = ctx.hash_build(torch.from_numpy(coords).cuda())
        k = ctx.kmap_subm3(h)
        w = torch.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(workloads.kaiming_normal_slat(c, c, 2)), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, w)
        x = torch.from_numpy(workloads.normal((n, c), 1)).cuda().to(torch.bfloat16)
        b = torch.from_numpy(workloads.normal((c,), 3, 0.1)).cuda()
        out = torch.empty((n, c), device="cuda")
        flags = s3dsp.CONV_TILE128 if a.case == "conv2" else s3dsp.CONV_STREAM_K
        for _ in range(1 + a.reps):
            ctx.conv(k, 27, P, x, w, b, out, c, flags=flags)
    elif a.case == "conv1_tf32":
        cfg = workloads.config1(0)
        coords, n, c = cfg["coords"], len(cfg["coords"]), 64
        k = ctx.kmap_subm3(ctx.hash_build(torch.from_numpy(coords).cuda()))
        P3 = s3dsp.PREC_F32_3XTF32
        w = torch.empty(s3dsp.Context.packed_bytes(P3, 27, c, c), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(cfg["weight"]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P3, w)
        x = torch.from_numpy(cfg["feats"]).cuda()
        b = torch.from_numpy(cfg["bias"]).cuda()
        out = torch.empty((n, c), device="cuda")
        for _ in range(1 + a.reps):
            ctx.conv(k, 27, P3, x, w, b, out, c)
    elif a.case == "coords":
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        bits = np.load(os.path.join(root, "tests", "golden", "ss_occ_mask.npz"))["bits"]
        grid = torch.from_numpy(np.unpackbits(bits)[: 64 ** 3].astype(np.float32).reshape(64, 64, 64)).cuda()
        bufs = [torch.empty((grid.numel(), 4), dtype=torch.int32, device="cuda") for _ in range(3)]
        for _ in range(1 + a.reps):
            m1 = ctx.occupancy_coords(grid, bufs[0])
            m2 = ctx.prune_surface(bufs[0][:m1], bufs[1])
            ctx.downsample_coords(bufs[1][:m2], bufs[2], 42000, 2, 42)
    elif a.case == "gs_tables":
        coords = torch.from_numpy(workloads.config2(seed=0)["coords"]).cuda()
        n = coords.shape[0]
        bkt = torch.empty(n, dtype=torch.int32, device="cuda")
        bwd = torch.empty(n, dtype=torch.int32, device="cuda")
        ape = torch.empty((n, 768), device="cuda")
        for _ in range(1 + a.reps):
            for si in (0, 1):
                ctx.gs_window_tables(coords, 4 * si, bkt, bwd)
            ctx.ape(coords, ape)
    elif a.case == "flexicubes":
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        t = np.load(os.path.join(root, "tests", "golden", "flexicubes_tables.npz"))
        tab = ctx.flexicubes_tables(t["dmc"], t["num_dual"], t["check"])
        coords, raw = workloads.flexicubes_input(64, 0)
        dc, dr = torch.from_numpy(coords).cuda(), torch.from_numpy(raw).cuda()
        for _ in range(1 + a.reps):
            ctx.flexicubes(tab, dr, dc).free()
    else:
        coords = workloads.ellipsoid_shell(512, 0, thickness=4.0)  # the config-5b volume
        d = torch.from_numpy(coords).cuda()
        for _ in range(1 + a.reps):
            h = ctx.hash_build(d)
            k = ctx.kmap_subm3(h)
            k.free()
            h.free()
    torch.cuda.synchronize()
    ctx.check()
    print(f"{a.case}: ok", flush=True)


if __name__ == "__main__":
    main()
