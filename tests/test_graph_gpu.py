"""A residual-block step captured as one CUDA graph and replayed.

Library kernels are launched with programmatic dependent launch: each may start
while the kernel before it finishes and waits (griddepcontrol.wait) before
touching global memory. In a captured graph those launches become programmatic
edges. The replays here get new input features between replays, and each
replay's output must equal, bit for bit, the eager step on the same input; a
kernel reading its predecessor's output too early would break that."""
import numpy as np
import pytest
import torch

import s3dsp
import workloads

pytestmark = pytest.mark.gpu


class Step:
    def __init__(self, ctx, cfg, c):
        P = s3dsp.PREC_BF16
        self.ctx, self.c = ctx, c
        n = len(cfg["coords"])
        self.n = n
        self.coords = torch.from_numpy(cfg["coords"]).cuda()
        self.x = torch.from_numpy(cfg["feats"]).cuda()
        self.w = []
        for key in ("w1", "w2"):
            dst = torch.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=torch.uint8, device="cuda")
            ctx.weights_pack(torch.from_numpy(cfg[key]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, dst)
            self.w.append(dst)
        self.b1, self.b2 = torch.from_numpy(cfg["b1"]).cuda(), torch.from_numpy(cfg["b2"]).cuda()
        self.gamma, self.beta = torch.from_numpy(cfg["gamma"]).cuda(), torch.from_numpy(cfg["beta"]).cuda()
        self.part = torch.empty(s3dsp.Context.gn_partials_count(n, c, 32), dtype=torch.float64, device="cuda")
        self.sub, self.mul, self.add = (torch.empty(c, device="cuda") for _ in range(3))
        self.xb = torch.empty((n, c), dtype=torch.bfloat16, device="cuda")
        self.y1 = torch.empty((n, c), dtype=torch.float32, device="cuda")
        self.hb = torch.empty((n, c), dtype=torch.bfloat16, device="cuda")
        self.out = torch.empty((n, c), dtype=torch.float32, device="cuda")

    def __call__(self):
        ctx, P = self.ctx, s3dsp.PREC_BF16
        h = ctx.hash_build(self.coords)
        k = ctx.kmap_subm3(h)
        ctx.convert(self.x, self.xb)
        ctx.conv(k, 27, P, self.xb, self.w[0], self.b1, self.y1, self.c, gn_partials=self.part, gn_groups=32)
        ctx.gn_finalize(self.part, self.n, self.c, 32, 1e-5, self.gamma, self.beta, self.sub, self.mul, self.add)
        ctx.channel_affine(self.y1, self.sub, self.mul, self.add, True, self.hb)
        ctx.conv(k, 27, P, self.hb, self.w[1], self.b2, self.out, self.c, residual=self.x)
        k.free()
        h.free()


@pytest.mark.parametrize("channels", [64, 256])
def test_graph_replays_match_eager(channels):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ctx = s3dsp.Context(0, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
        step = Step(ctx, workloads.config2(seed=0, channels=channels), channels)
        inputs = [torch.from_numpy(workloads.normal((step.n, channels), 500 + i)).cuda() for i in range(3)]
        expected = []
        for x in inputs:
            step.x.copy_(x)
            step()
            expected.append(step.out.clone())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
            step()
        for rep in range(2):
            for x, e in zip(inputs, expected):
                step.out.fill_(float("nan"))
                step.x.copy_(x)
                graph.replay()
                stream.synchronize()
                assert torch.equal(step.out, e), f"replay {rep}: output differs from the eager step"
        del graph
        ctx.check()
    assert np.isfinite(expected[0].cpu().numpy()).all()
