"""Independent contexts used concurrently from several host threads.

The C ABI promises that separate contexts (each on its own stream) may run at
the same time, as the reference's handles may. Every thread here runs whole
host-buffer residual blocks (upload, hash, kernel map, two convolutions,
GroupNorm, download) on its own object; each output must equal, bit for bit,
the same call made alone on one context. The kernels are deterministic (no
float atomics on outputs, fixed-order GroupNorm partials), so any sharing of
scratch or state between contexts would show up as a difference."""
import threading

import numpy as np
import pytest
import torch

import s3dsp
import workloads

pytestmark = pytest.mark.gpu

THREADS, CALLS, C = 4, 3, 64


def pinned(a):
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


@pytest.fixture(scope="module")
def setup():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    ctx = s3dsp.Context(0)
    P = s3dsp.PREC_BF16
    w = workloads.config2(seed=0, channels=C)
    packs = []
    for key in ("w1", "w2"):
        dst = torch.empty(s3dsp.Context.packed_bytes(P, 27, C, C), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(w[key]), s3dsp.LAYOUT_SLAT_ROW, 27, C, C, P, dst)
        packs.append(dst)
    params = dict(w1=packs[0], w2=packs[1], b1=torch.from_numpy(w["b1"]).cuda(), b2=torch.from_numpy(w["b2"]).cuda(),
                  gamma=torch.from_numpy(w["gamma"]).cuda(), beta=torch.from_numpy(w["beta"]).cuda())
    # one object per thread: different shells and features
    objs = []
    for t in range(THREADS):
        coords = workloads.ellipsoid_shell(32 + 8 * t, t)
        objs.append((pinned(coords), pinned(workloads.normal((len(coords), C), 100 + t))))
    torch.cuda.synchronize()
    expected = []
    for coords, x in objs:
        out = torch.empty((coords.shape[0], C), dtype=torch.float32).pin_memory()
        ctx.res_block_gn_host(P, coords, x, params["w1"], params["b1"], params["gamma"], params["beta"],
                              params["w2"], params["b2"], out)
        expected.append(out.clone())
    return params, objs, expected


@pytest.mark.parametrize("flags", [0, s3dsp.CONTEXT_DEFERRED_CHECKS])
def test_concurrent_host_blocks_bit_exact(setup, flags):
    params, objs, expected = setup
    errors, results = [], [None] * THREADS
    start = threading.Barrier(THREADS)

    def body(t):
        try:
            torch.cuda.set_device(0)
            st = torch.cuda.Stream()
            cx = s3dsp.Context(0, stream=st.cuda_stream, flags=flags)
            coords, x = objs[t]
            outs = [torch.empty((coords.shape[0], C), dtype=torch.float32).pin_memory() for _ in range(CALLS)]
            start.wait()
            for o in outs:
                cx.res_block_gn_host(s3dsp.PREC_BF16, coords, x, params["w1"], params["b1"], params["gamma"],
                                     params["beta"], params["w2"], params["b2"], o)
            cx.check()
            results[t] = outs
        except Exception as e:  # reported below
            errors.append(e)
            start.abort()

    threads = [threading.Thread(target=body, args=(t,)) for t in range(THREADS)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for t in range(THREADS):
        for o in results[t]:
            assert torch.equal(o, expected[t]), f"thread {t}: output differs from the call made alone"


def test_queued_host_blocks_round_robin_bit_exact(setup):
    """One host thread queues host-buffer blocks on several contexts
    (s3dsp_res_block_gn_host_queued), round robin; after the streams drain,
    every output equals the synchronous call's, bit for bit."""
    params, objs, expected = setup
    lanes = []
    for t in range(THREADS):
        st = torch.cuda.Stream()
        lanes.append((st, s3dsp.Context(0, stream=st.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)))
    outs = [[torch.empty((objs[t][0].shape[0], C), dtype=torch.float32).pin_memory() for _ in range(CALLS)]
            for t in range(THREADS)]
    for i in range(CALLS):
        for t, (st, cx) in enumerate(lanes):
            coords, x = objs[t]
            cx.res_block_gn_host_queued(s3dsp.PREC_BF16, coords, x, params["w1"], params["b1"], params["gamma"],
                                        params["beta"], params["w2"], params["b2"], outs[t][i])
    for st, cx in lanes:
        st.synchronize()
        cx.check()
    for t in range(THREADS):
        for o in outs[t]:
            assert torch.equal(o, expected[t]), f"context {t}: queued output differs from the synchronous call's"


def test_copy_stream_host_blocks_bit_exact(setup):
    """A context with copy streams (CONTEXT_COPY_STREAMS) pipelines queued
    host-buffer blocks over its three staging slots: one call's upload, the
    next one's kernels and the previous one's download overlap. Objects of
    four sizes in turn make the slots grow (and then serve smaller calls);
    after check (which joins the copy streams) every output equals the
    synchronous call's on a plain context, bit for bit, and so does a
    synchronous call on the same context."""
    params, objs, expected = setup
    st = torch.cuda.Stream()
    cx = s3dsp.Context(0, stream=st.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS | s3dsp.CONTEXT_COPY_STREAMS)
    order = [0, 1, 2, 3, 3, 2, 1, 0, 0, 2, 1, 3]  # every slot reused several times
    outs = [torch.empty((objs[t][0].shape[0], C), dtype=torch.float32).pin_memory() for t in order]
    cx.fork()
    for j, t in enumerate(order):
        coords, x = objs[t]
        cx.res_block_gn_host_queued(s3dsp.PREC_BF16, coords, x, params["w1"], params["b1"], params["gamma"],
                                    params["beta"], params["w2"], params["b2"], outs[j])
    cx.check()
    for j, t in enumerate(order):
        assert torch.equal(outs[j], expected[t]), f"call {j} (object {t}): output differs from the synchronous call's"
    coords, x = objs[2]
    out = torch.empty((coords.shape[0], C), dtype=torch.float32).pin_memory()
    cx.res_block_gn_host(s3dsp.PREC_BF16, coords, x, params["w1"], params["b1"], params["gamma"], params["beta"],
                         params["w2"], params["b2"], out)
    assert torch.equal(out, expected[2])
    cx.close()
    plain = s3dsp.Context(0)
    plain.fork()  # no copy streams: both are no-ops
    plain.join()


def test_queued_host_block_needs_deferred_checks(setup):
    params, objs, _ = setup
    cx = s3dsp.Context(0)
    coords, x = objs[0]
    out = torch.empty((coords.shape[0], C), dtype=torch.float32).pin_memory()
    with pytest.raises(s3dsp.S3dError) as ei:
        cx.res_block_gn_host_queued(s3dsp.PREC_BF16, coords, x, params["w1"], params["b1"], params["gamma"],
                                    params["beta"], params["w2"], params["b2"], out)
    assert ei.value.status == s3dsp.S3D_INVALID_ARGUMENT
