"""The SLat Gaussian decoder's Swin torso over the s3dsp C ABI.

gs_decoder_graph.cpp:13-155:

  input_layer   Linear 8 -> 768, + the absolute position embedding (:37-48)
  12 blocks     h1 = LayerNorm(h) (1e-6, no affine) gathered to bucket order
                (the window tables of shift 0 for even blocks, (4,4,4) for odd);
                q, k, v = Linear 768 -> 3 x 768; per Swin window and head
                softmax(q k^T / sqrt(64)) v; back to token order; Linear 768 ->
                768; h += it (:55-125); then h += Linear 3072 -> 768 (GELU(
                Linear 768 -> 3072 (LayerNorm(h)))) (:127-142)
  final         LayerNorm (1e-5, no affine) -> out_layer Linear 768 -> 448 (:146-151)

The window tables and the APE come from s3dsp_gs_window_tables / s3dsp_ape
(GsTables::build, sparse_ops.cpp:182-270); the Linears are s3dsp_conv with
no kernel map (the residual adds and the GELU in their epilogues), the
attention s3dsp_window_attention (f32), the bucket-order gather
s3dsp_gather_rows. Weights are random (seeded) with the reference's shapes.
"""
from __future__ import annotations

import numpy as np

import workloads

IN_CH, C, HEADS, MLP, OUT_CH, BLOCKS, WINDOW = 8, 768, 12, 3072, 448, 12, 8


def gs_params(seed: int = 0, blocks: int = BLOCKS) -> dict:
    """Seeded random parameters, Linears (Cout, Cin) as gb_linear takes them."""
    s = 1000 * seed

    def lin(cout, cin, k):
        return dict(w=workloads.normal((cout, cin), s + k, float(np.sqrt(1.0 / cin))),
                    b=workloads.normal((cout,), s + k + 1, 0.02))

    p = {"input_layer": lin(C, IN_CH, 1), "out_layer": lin(OUT_CH, C, 3)}
    p["blocks"] = [dict(qkv=lin(3 * C, C, 100 + 10 * i), out=lin(C, C, 102 + 10 * i),
                        mlp0=lin(MLP, C, 104 + 10 * i), mlp2=lin(C, MLP, 106 + 10 * i)) for i in range(blocks)]
    return p


def units(n: int, blocks: int = BLOCKS) -> int:
    """Output token rows of every Linear and of the attention in one pass."""
    return n * (2 + 5 * blocks)  # input, out layer; per block qkv, attention, out, mlp0, mlp2


class GsTablesDev:
    """Both shifts' window tables on the device, the windows as (first row,
    rows) pairs, and the 768-channel APE."""

    def __init__(self, s3dsp, ctx, coords, torch):
        n = coords.shape[0]
        self.n = n
        dev = coords.device
        self.bkt, self.windows, self.buckets = [], [], []
        for si in (0, 1):
            bkt = torch.empty(n, dtype=torch.int32, device=dev)
            bwd = torch.empty(n, dtype=torch.int32, device=dev)
            b = ctx.gs_window_tables(coords, 4 * si, bkt, bwd, WINDOW)
            win = np.concatenate([np.stack([off + len_ * np.arange(nw), np.full(nw, len_)], axis=1)
                                  for len_, off, nw in b]).astype(np.int32) if len(b) else np.zeros((0, 2), np.int32)
            self.bkt.append(bkt)
            self.windows.append(torch.from_numpy(np.ascontiguousarray(win)).to(dev))
            self.buckets.append(b)
        self.ape = torch.empty((n, C), dtype=torch.float32, device=dev)
        ctx.ape(coords, self.ape)


class GsTorso:
    """The torso on one device; Linear weights packed once for `precision`
    (the attention runs in f32 at every precision)."""

    def __init__(self, s3dsp, ctx, params: dict, precision: int, device):
        import torch
        self.s, self.ctx, self.torch, self.prec, self.dev = s3dsp, ctx, torch, precision, device
        self.act = torch.bfloat16 if precision == s3dsp.PREC_BF16 else torch.float32

        def lin(d):
            w = np.ascontiguousarray(d["w"], dtype=np.float32)
            cout, cin = w.shape
            dst = torch.empty(s3dsp.Context.packed_bytes(precision, 1, cin, cout), dtype=torch.uint8, device=device)
            ctx.weights_pack(torch.from_numpy(w), s3dsp.LAYOUT_LINEAR, 1, cin, cout, precision, dst)
            return dst, torch.from_numpy(np.ascontiguousarray(d["b"], dtype=np.float32)).to(device), cout

        self.lin_in = lin(params["input_layer"])
        self.lin_out = lin(params["out_layer"])
        self.blocks = [{k: lin(v) for k, v in b.items()} for b in params["blocks"]]

    def _act(self, x):
        """x in the dtype the Linears read (bf16 for BF16)."""
        if x.dtype == self.act:
            return x
        y = self.torch.empty(x.shape, dtype=self.act, device=self.dev)
        self.ctx.convert(x, y)
        return y

    def _linear(self, x, wbc, residual=None, flags=0, out_dtype=None):
        t = self.torch
        w, b, cout = wbc
        out = t.empty((x.shape[0], cout), dtype=out_dtype or t.float32, device=self.dev)
        self.ctx.conv(None, 1, self.prec, self._act(x), w, b, out, cout, residual=residual, flags=flags)
        return out

    def forward(self, tb: GsTablesDev, x, taps=None):
        """x: f32 [n, 8] -> f32 [n, 448]."""
        t, ctx, s = self.torch, self.ctx, self.s
        n = tb.n
        h = self._linear(x, self.lin_in, residual=tb.ape)
        for i, blk in enumerate(self.blocks):
            si = i % 2
            h1 = t.empty((n, C), dtype=self.act, device=self.dev)
            ctx.layer_norm(h, 1e-6, h1)
            hb = t.empty_like(h1)
            ctx.gather_rows(h1, tb.bkt[si], hb)
            qkv = self._linear(hb, blk["qkv"])
            ao = t.empty((n, C), dtype=t.float32, device=self.dev)
            ctx.window_attention(qkv, HEADS, tb.windows[si], ao, scatter=tb.bkt[si])
            h = self._linear(ao, blk["out"], residual=h)
            h2 = t.empty((n, C), dtype=self.act, device=self.dev)
            ctx.layer_norm(h, 1e-6, h2)
            g = self._linear(h2, blk["mlp0"], flags=s.EPI_GELU, out_dtype=self.act)
            h = self._linear(g, blk["mlp2"], residual=h)
            if taps is not None:
                taps[f"block{i}"] = h
        hn = t.empty((n, C), dtype=self.act, device=self.dev)
        ctx.layer_norm(h, 1e-5, hn)
        return self._linear(hn, self.lin_out)
