"""Config 4: a mesh-decoder-shaped stack over the s3dsp C-ABI.

latent (8 channels) on the active voxels of a 64^3 object
  -> Linear 8 -> 256
  -> 4 GroupNorm residual blocks at C = 256     (s3dsp_res_block_gn)
  -> subdivide to 128^3, C = 128                 (s3dsp_mesh_upsample_level)
  -> 2 residual blocks at C = 128
  -> subdivide to 256^3, C = 64
  -> 2 residual blocks at C = 64
  -> Linear 64 -> 32
The subdivide levels are MeshUpsampleGraph::build (mesh_decoder_graph.cpp:
42-132: GN, SiLU, repeat_children, conv, GN, SiLU, conv, + 1x1 skip); the
residual blocks are the config-2 block (conv3, GN(32), SiLU, conv3, + x);
the linears are gb_linear (graph_builder.cpp:44-54). Every subdivide keeps
all 8 children (MeshSubdivideTables semantics), so rows grow 64x overall.

Weights are random (seeded): the stack has the reference decoder's shape, not
its trained parameters.
"""
from __future__ import annotations

import numpy as np

import workloads

WIDTHS = (256, 128, 64)
BLOCKS = (4, 2, 2)
LATENT, HEAD = 8, 32


def _block(c, seed):
    return dict(w1=workloads.conv_weight_slat(c, c, seed), b1=workloads.normal((c,), seed + 1, 0.05),
                gamma=workloads.normal((c,), seed + 2, 0.1) + 1.0, beta=workloads.normal((c,), seed + 3, 0.05),
                w2=workloads.conv_weight_slat(c, c, seed + 4), b2=workloads.normal((c,), seed + 5, 0.05))


def _level(cin, cout, seed):
    return dict(gn1_w=workloads.normal((cin,), seed, 0.1) + 1.0, gn1_b=workloads.normal((cin,), seed + 1, 0.05),
                conv1_w=workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cin, cout, seed + 2), cin, cout),
                conv1_b=workloads.normal((cout,), seed + 3, 0.05),
                gn2_w=workloads.normal((cout,), seed + 4, 0.1) + 1.0, gn2_b=workloads.normal((cout,), seed + 5, 0.05),
                conv2_w=workloads.slat_to_mesh_packed(workloads.conv_weight_slat(cout, cout, seed + 6), cout, cout),
                conv2_b=workloads.normal((cout,), seed + 7, 0.05),
                skip_w=workloads.normal((1, cout * cin), seed + 8, float(np.sqrt(1.0 / cin))),
                skip_b=workloads.normal((cout,), seed + 9, 0.05))


def config4_params(seed: int = 0) -> dict:
    """Seeded random parameters of the whole stack (numpy, reference layouts:
    SLat conv (Cout, 27, Cin), mesh conv packed (27, Cout*Cin), Linear (Cout, Cin))."""
    s = 1000 * seed
    p = {"lin_in": dict(w=workloads.normal((WIDTHS[0], LATENT), s + 1, float(np.sqrt(1.0 / LATENT))),
                        b=workloads.normal((WIDTHS[0],), s + 2, 0.05)),
         "lin_out": dict(w=workloads.normal((HEAD, WIDTHS[-1]), s + 3, float(np.sqrt(1.0 / WIDTHS[-1]))),
                         b=workloads.normal((HEAD,), s + 4, 0.05))}
    for lv, (c, nb) in enumerate(zip(WIDTHS, BLOCKS)):
        p[f"blocks{lv}"] = [_block(c, s + 100 * (lv + 1) + 10 * i) for i in range(nb)]
        if lv + 1 < len(WIDTHS):
            p[f"up{lv + 1}"] = _level(c, WIDTHS[lv + 1], s + 500 + 20 * lv)
    return p


def units(n: int) -> int:
    """Output voxel rows of every conv / linear layer of one forward over an
    object of n voxels: the stack's unit of work (one output voxel of one layer)."""
    rows, total = n, n  # input linear
    for lv, nb in enumerate(BLOCKS):
        total += 2 * nb * rows  # two convs per residual block
        if lv + 1 < len(BLOCKS):
            rows *= 8
            total += 3 * rows  # conv1, conv2 and the 1x1 skip of the subdivide level
    return total + rows  # output linear


class Config4Stack:
    """The stack on one device; weights packed once for `precision`."""

    def __init__(self, s3dsp, ctx, params: dict, precision: int, device):
        import torch
        self.s, self.ctx, self.torch, self.prec, self.dev = s3dsp, ctx, torch, precision, device

        def dev(a):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)

        def pack(w, layout, kvol, cin, cout):
            dst = torch.empty(s3dsp.Context.packed_bytes(precision, kvol, cin, cout), dtype=torch.uint8, device=device)
            ctx.weights_pack(torch.from_numpy(np.ascontiguousarray(w, dtype=np.float32)), layout, kvol, cin, cout,
                             precision, dst)
            return dst

        L = s3dsp
        self.lin_in = (pack(params["lin_in"]["w"], L.LAYOUT_LINEAR, 1, LATENT, WIDTHS[0]), dev(params["lin_in"]["b"]))
        self.lin_out = (pack(params["lin_out"]["w"], L.LAYOUT_LINEAR, 1, WIDTHS[-1], HEAD), dev(params["lin_out"]["b"]))
        self.blocks, self.ups = [], []
        for lv, c in enumerate(WIDTHS):
            self.blocks.append([dict(w1=pack(b["w1"], L.LAYOUT_SLAT_ROW, 27, c, c), b1=dev(b["b1"]),
                                     gamma=dev(b["gamma"]), beta=dev(b["beta"]),
                                     w2=pack(b["w2"], L.LAYOUT_SLAT_ROW, 27, c, c), b2=dev(b["b2"]))
                                for b in params[f"blocks{lv}"]])
            if lv + 1 < len(WIDTHS):
                u, co = params[f"up{lv + 1}"], WIDTHS[lv + 1]
                self.ups.append(dict(gn1_w=dev(u["gn1_w"]), gn1_b=dev(u["gn1_b"]),
                                     conv1_w=pack(u["conv1_w"], L.LAYOUT_MESH_PACKED, 27, c, co),
                                     conv1_b=dev(u["conv1_b"]), gn2_w=dev(u["gn2_w"]), gn2_b=dev(u["gn2_b"]),
                                     conv2_w=pack(u["conv2_w"], L.LAYOUT_MESH_PACKED, 27, co, co),
                                     conv2_b=dev(u["conv2_b"]),
                                     skip_w=pack(u["skip_w"].reshape(co, c), L.LAYOUT_LINEAR, 1, c, co),
                                     skip_b=dev(u["skip_b"])))

    def _linear(self, x, wb, cout):
        t, s = self.torch, self.s
        if self.prec == s.PREC_BF16:
            xb = t.empty(x.shape, dtype=t.bfloat16, device=self.dev)
            self.ctx.convert(x, xb)
            x = xb
        out = t.empty((x.shape[0], cout), dtype=t.float32, device=self.dev)
        self.ctx.conv(None, 1, self.prec, x, wb[0], wb[1], out, cout)
        return out

    def forward(self, coords, latent):
        """coords: device int32 [N, 4]; latent: device f32 [N, 8]. Returns the
        final child coordinates [64N, 4] and the head output f32 [64N, 32]."""
        t, ctx = self.torch, self.ctx
        x = self._linear(latent, self.lin_in, WIDTHS[0])
        h = ctx.hash_build(coords, reject_duplicates=True)
        for lv, c in enumerate(WIDTHS):
            k = ctx.kmap_subm3(h)
            for b in self.blocks[lv]:
                y = t.empty_like(x)
                ctx.res_block_gn(k, self.prec, x, b["w1"], b["b1"], b["gamma"], b["beta"], b["w2"], b["b2"], y)
                x = y
            k.free()
            if lv + 1 < len(WIDTHS):
                u, co = self.ups[lv], WIDTHS[lv + 1]
                coords = t.empty((8 * x.shape[0], 4), dtype=t.int32, device=self.dev)
                y = t.empty((8 * x.shape[0], co), dtype=t.float32, device=self.dev)
                ctx.mesh_upsample_level(h, self.prec, x, co, u["gn1_w"], u["gn1_b"], u["conv1_w"], u["conv1_b"],
                                        u["gn2_w"], u["gn2_b"], u["conv2_w"], u["conv2_b"], u["skip_w"], u["skip_b"],
                                        coords, y)
                h.free()
                h = ctx.hash_build(coords, reject_duplicates=True)
                x = y
        h.free()
        return coords, self._linear(x, self.lin_out, HEAD)
