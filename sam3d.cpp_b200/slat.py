"""The SLat flow generator's sparse stages over the s3dsp C ABI.

One flow step of the structured-latent generator (slat_flow_graph.cpp) has a
sparse half around a dense transformer torso:

  input_layer     Linear 8 -> 128 on the nf fine voxels              (:283-285)
  input_blocks.0  res_block 128 -> 128, fine map                      (:290-291)
  input_blocks.1  2x mean-pool to the nc coarse voxels, res_block
                  128 -> 1024 on the coarse map, Linear skip          (:294-296)
  -- APE + transformer blocks on the coarse rows (dense; the caller's) --
  out_blocks.0    concat(h, skip1) 2048 coarse -> nearest upsample ->
                  res_block 2048 -> 128 on the fine map, Linear skip (:463-495)
  out_blocks.1    concat(h, skip0) 256 fine -> res_block 256 -> 128,
                  Linear skip                                         (:496-524)
  final           LayerNorm (no affine) -> out_layer Linear 128 -> 8  (:527-531)

A res_block is LayerNorm(1e-6, affine) -> SiLU -> conv1 -> LayerNorm(1e-6)
-> h * (1 + scale) + shift -> SiLU -> conv2 -> + skip (:216-275). Its
scale / shift come from the timestep embedding through the block's
emb_layers (a dense Linear per flow step): they are the caller's input here,
`mods[block] = (scale [cout], shift [cout])`.

The concats are never built: norm1 and the convs read the two sources
directly (s3dsp_layer_norm_concat, s3dsp_conv_concat), and the upsampled
2048-wide rows of out_blocks.0 are never built either: norm1 and the skip
Linear run on the coarse rows (both row-wise), conv1 gathers coarse rows
through the fine map composed with fine_to_coarse
(s3dsp_slat_res_block_concat with up_rows).

Weights are random (seeded) with the reference's shapes and GGUF layouts.
"""
from __future__ import annotations

import numpy as np

import workloads

IN_CH, IO_CH, MODEL_CH, OUT_CH = 8, 128, 1024, 8
BLOCKS = {  # name: (cin_a, cin_b, cout)
    "input_blocks.0": (IO_CH, 0, IO_CH),
    "input_blocks.1": (IO_CH, 0, MODEL_CH),
    "out_blocks.0": (MODEL_CH, MODEL_CH, IO_CH),
    "out_blocks.1": (IO_CH, IO_CH, IO_CH),
}


def _block_params(cin, cout, seed):
    p = dict(norm1_w=workloads.normal((cin,), seed, 0.1) + 1.0, norm1_b=workloads.normal((cin,), seed + 1, 0.05),
             conv1_w=workloads.conv_weight_slat(cin, cout, seed + 2), conv1_b=workloads.normal((cout,), seed + 3, 0.05),
             conv2_w=workloads.conv_weight_slat(cout, cout, seed + 4),
             conv2_b=workloads.normal((cout,), seed + 5, 0.05))
    if cin != cout:
        p["skip_w"] = workloads.normal((cout, cin), seed + 6, float(np.sqrt(1.0 / cin)))
        p["skip_b"] = workloads.normal((cout,), seed + 7, 0.05)
    return p


def slat_params(seed: int = 0) -> dict:
    """Seeded random parameters in the reference layouts: conv weights
    (Cout, 27 * Cin) (SLat row layout), Linears (Cout, Cin)."""
    s = 1000 * seed
    p = {"input_layer": dict(w=workloads.normal((IO_CH, IN_CH), s + 1, float(np.sqrt(1.0 / IN_CH))),
                             b=workloads.normal((IO_CH,), s + 2, 0.05)),
         "out_layer": dict(w=workloads.normal((OUT_CH, IO_CH), s + 3, float(np.sqrt(1.0 / IO_CH))),
                           b=workloads.normal((OUT_CH,), s + 4, 0.05))}
    for i, (name, (ca, cb, co)) in enumerate(BLOCKS.items()):
        p[name] = _block_params(ca + cb, co, s + 100 * (i + 1))
    return p


def slat_mods(seed: int = 0) -> dict:
    """Stand-ins for each block's adaLN (scale, shift) of one flow step."""
    return {name: (workloads.normal((co,), 7000 + 10 * i + seed, 0.1),
                   workloads.normal((co,), 7001 + 10 * i + seed, 0.1))
            for i, (name, (_, _, co)) in enumerate(BLOCKS.items())}


def units(nf: int, nc: int) -> int:
    """Output voxel rows of every conv / linear layer of one sparse pass: the
    unit of work (one output voxel of one layer)."""
    return (nf            # input_layer
            + 2 * nf      # input_blocks.0 conv1, conv2
            + 3 * nc      # input_blocks.1 conv1, conv2, skip
            + 3 * nf      # out_blocks.0 conv1, conv2, skip (skip rows computed at nc, gathered to nf)
            + 3 * nf      # out_blocks.1
            + nf)         # out_layer


class SlatTablesDev:
    """Per-object tables on the device: fine hash and map, the coarse tables
    and map (SlatTables::build, sparse_ops.cpp:49-173), fine_to_coarse."""

    def __init__(self, s3dsp, ctx, coords, torch):
        self.hash = ctx.hash_build(coords)
        self.fine = ctx.kmap_subm3(self.hash)
        self.tables = ctx.slat_tables(self.hash)
        self.nf, self.nc = self.tables.nf, self.tables.nc
        self.coarse = self.tables.coarse_kmap
        self.f2c = torch.empty(self.nf, dtype=torch.int32, device=coords.device)
        ctx.slat_tables_export(self.tables, f2c=self.f2c)

    def free(self):
        self.tables.free()
        self.fine.free()
        self.hash.free()


class SlatSparse:
    """The sparse stages on one device; weights packed once for `precision`."""

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
        self.lin_in = (pack(params["input_layer"]["w"], L.LAYOUT_LINEAR, 1, IN_CH, IO_CH),
                       dev(params["input_layer"]["b"]))
        self.lin_out = (pack(params["out_layer"]["w"], L.LAYOUT_LINEAR, 1, IO_CH, OUT_CH),
                        dev(params["out_layer"]["b"]))
        self.blocks = {}
        for name, (ca, cb, co) in BLOCKS.items():
            b = params[name]
            ci = ca + cb
            d = dict(norm1_w=dev(b["norm1_w"]), norm1_b=dev(b["norm1_b"]),
                     conv1_w=pack(b["conv1_w"], L.LAYOUT_SLAT_ROW, 27, ci, co), conv1_b=dev(b["conv1_b"]),
                     conv2_w=pack(b["conv2_w"], L.LAYOUT_SLAT_ROW, 27, co, co), conv2_b=dev(b["conv2_b"]),
                     skip_w=None, skip_b=None)
            if "skip_w" in b:
                d["skip_w"] = pack(b["skip_w"], L.LAYOUT_LINEAR, 1, ci, co)
                d["skip_b"] = dev(b["skip_b"])
            self.blocks[name] = d

    def mods_to_device(self, mods: dict) -> dict:
        t = self.torch
        return {k: (t.from_numpy(np.ascontiguousarray(a)).to(self.dev), t.from_numpy(np.ascontiguousarray(b)).to(
            self.dev)) for k, (a, b) in mods.items()}

    def _linear(self, x, wb, cout):
        t, s = self.torch, self.s
        if self.prec == s.PREC_BF16:
            xb = t.empty(x.shape, dtype=t.bfloat16, device=self.dev)
            self.ctx.convert(x, xb)
            x = xb
        out = t.empty((x.shape[0], cout), dtype=t.float32, device=self.dev)
        self.ctx.conv(None, 1, self.prec, x, wb[0], wb[1], out, cout)
        return out

    def _block(self, name, kmap, xa, xb, mods, n_out, up_rows=None):
        b, co = self.blocks[name], BLOCKS[name][2]
        out = self.torch.empty((n_out, co), dtype=self.torch.float32, device=self.dev)
        sc, sh = mods[name]
        self.ctx.slat_res_block_concat(kmap, self.prec, xa, xb, co, b["norm1_w"], b["norm1_b"], b["conv1_w"],
                                       b["conv1_b"], sc, sh, b["conv2_w"], b["conv2_b"], b["skip_w"], b["skip_b"],
                                       out, up_rows=up_rows)
        return out

    def encode(self, tb: SlatTablesDev, x, mods):
        """x: f32 [nf, 8] -> (skip0 [nf, 128], skip1 [nc, 1024])."""
        t = self.torch
        h = self._linear(x, self.lin_in, IO_CH)
        skip0 = self._block("input_blocks.0", tb.fine, h, None, mods, tb.nf)
        d = t.empty((tb.nc, IO_CH), dtype=t.float32, device=self.dev)
        self.ctx.slat_downsample(tb.tables, skip0, d)
        skip1 = self._block("input_blocks.1", tb.coarse, d, None, mods, tb.nc)
        return skip0, skip1

    def decode(self, tb: SlatTablesDev, h, skip0, skip1, mods):
        """h: f32 [nc, 1024] (the transformer torso's output) -> f32 [nf, 8]."""
        t = self.torch
        h = self._block("out_blocks.0", tb.fine, h, skip1, mods, tb.nf, up_rows=tb.f2c)
        h = self._block("out_blocks.1", tb.fine, h, skip0, mods, tb.nf)
        hn = t.empty_like(h)
        self.ctx.layer_norm(h, 1e-6, hn)
        return self._linear(hn, self.lin_out, OUT_CH)

    def forward(self, tb: SlatTablesDev, x, mods, mid=None):
        """encode -> mid (the dense torso; identity when None) -> decode."""
        skip0, skip1 = self.encode(tb, x, mods)
        h = skip1 if mid is None else mid(skip1)
        return self.decode(tb, h, skip0, skip1, mods)
