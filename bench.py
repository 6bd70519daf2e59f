"""Benchmark of the sparse-convolution hot path (config 2: the residual block on a 64^3 shell at C = 256).

Workload (one "step" = one pass of the whole path over one object): the
64^3 ellipsoid-shell active set (seed 0), C = 256:
  coordinate hash -> submanifold kernel map -> subm conv3 (+ GroupNorm partial
  sums) -> GroupNorm(32) finalize -> SiLU -> subm conv3 -> + skip,
bf16 tcgen05 MMAs with f32 accumulation. Metric: active-voxel outputs/s, one
unit = one output voxel of one conv layer (2 * N per step); `value` is the
whole job's rate (all GPUs), `value_per_gpu` divides it by the GPU count.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload ...] [--no-sub] [--profile-case CASE]

Multi-GPU (torchrun, one rank per GPU): objects are independent, so each rank
runs its own object (seed = rank) with no data-path collective ("weak"
scaling); timing is the max over ranks.

The default run also measures, at every N, three sub-records on the same
ranks: `f32` (the config-2 step in the reference's own f32 arithmetic: F32
strict FFMA and 3xTF32 on the tensor cores), `objects_5a` (64 objects through
the config-4 stack, dealt to the ranks) and `volume_5b` (one 2.58M-voxel
volume in Morton slabs with the C-ABI NCCL halo exchange, checked bit for bit
against the whole-volume conv on every rank). `--no-sub` skips them.

`--impl reference` times the reference path on the host cores instead: the
reference's own table builder (oracle/_ref, when it was built) plus the CPU
restatement of its GGML op order, all host threads.

`--profile-case CASE` runs one small kernel case for an ncu capture and exits.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for sub in ("sam3d.cpp_b200", "oracle"):
    sys.path.insert(0, os.path.join(ROOT, sub))

METRIC = "active-voxel outputs/s, all GPUs (C=256 subm conv residual block)"
UNIT = "voxel-outputs/s"
L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2
E2E_FLUSH_BYTES = 256 << 20  # twice the L2: the flush inside the e2e timed region
# DRAM bytes (read + write) per launch, from one ncu capture of
# `python bench.py --profile-case conv2` (128-row kernel) and of
# `--profile-case conv2_pairs` (the dispatched split-K pair kernel), keyed by
# (kernel, output rows, channels): each holds only for that kernel on that
# shape; other shapes report null until captured.
CONV_TRAFFIC_BYTES = {("conv_tc_kernel", 15159, 256): 13.02e6, ("conv_sk_kernel<256>:pairs", 15159, 256): 13.09e6}
FFMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal FP32 FMA peak of B200 (148 SMs x 128 lanes x 2 x 1.965 GHz)


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return pk["hbm_gbs"], pk["bf16_tflops"], pk.get("bf16_tflops_sustained"), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region (recipe's clocks line)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_cpus(local_rank: int, local_world: int):
    """Host CPUs for this rank: the NUMA node of its GPU (from sysfs), shared
    evenly among the ranks of this host on that node (by local rank). None
    when the node cannot be found."""
    import torch
    try:
        pr = torch.cuda.get_device_properties(local_rank)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None

        def node_of(i):
            q = torch.cuda.get_device_properties(i)
            b = f"{q.pci_domain_id:04x}:{q.pci_bus_id:02x}:{q.pci_device_id:02x}.0"
            with open(f"/sys/bus/pci/devices/{b}/numa_node") as g:
                return int(g.read().strip())

        peers = [i for i in range(local_world) if node_of(i) == node]
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = []
            for part in f.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.extend(range(int(lo), int(hi or lo) + 1))
        cpus = [c for c in cpus if c in os.sched_getaffinity(0)]
        share = len(cpus) // max(1, len(peers))
        if share < 1:
            return None
        i = peers.index(local_rank)
        return cpus[i * share:(i + 1) * share]
    except Exception:
        return None


def conv_roofline(kernel, n, c, P, conv_ms, out_bytes, res_bytes, tflops, hbm, peak_src):
    """North_star's roofline for one conv launch: the slower of the dense MMA
    time (2 C^2 P at the measured bf16 peak) and the gathered bytes at HBM
    bandwidth (P gathered rows of C bf16 + N output rows + the residual rows
    read + 8 bytes of pair indices per pair + the 27 C^2 bf16 weights).
    `achieved` follows the binding side; the other side is reported beside it."""
    flops = 2.0 * c * c * P
    gbytes = P * c * 2 + n * c * out_bytes + n * c * res_bytes + 8 * P + 27 * c * c * 2
    t_mma, t_hbm = flops / (tflops * 1e12), gbytes / (hbm * 1e9)
    s = conv_ms / 1e3
    tensor = {"achieved": flops / s / 1e12, "peak": tflops, "unit": "TFLOP/s", "frac": flops / s / 1e12 / tflops}
    hbm_v = {"achieved": gbytes / s / 1e9, "peak": hbm, "unit": "GB/s", "frac": gbytes / s / 1e9 / hbm}
    bound = "tensor" if t_mma >= t_hbm else "hbm"
    main, other = (tensor, hbm_v) if bound == "tensor" else (hbm_v, tensor)
    key = (kernel, n, c)
    return {"bound": bound, **main, "traffic": CONV_TRAFFIC_BYTES.get(key),
            "traffic_unit": "DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum), measured for "
                            "this (kernel, rows, channels) only",
            "kernel": kernel, "flops_per_launch": flops, "gathered_bytes_per_launch": gbytes,
            "avg_launch_ms": conv_ms, "roofline_ms": max(t_mma, t_hbm) * 1e3,
            ("tensor_view" if bound == "hbm" else "hbm_view"): other,
            "peak_source": f"{peak_src} MEASURED_PEAKS.json (bf16_tflops burst, hbm_gbs)"}


# ---------------------------------------------------------------------------
# our path
# ---------------------------------------------------------------------------
class ResBlockPath:
    """Config-2 residual block through the s3dsp C-ABI (device-resident).

    BF16: x is converted to bf16 on a side stream (its own context) while the
    hash and kernel map are built; conv1 writes y1 in bf16 with the GroupNorm
    partial sums taken from its f32 accumulators; GN + SiLU read y1 and write
    the bf16 input of conv2, which adds the f32 skip. F32 precisions (strict
    FFMA, 3xTF32) keep every activation in f32, the reference's arithmetic."""

    PHASES = ("hash+kmap", "conv1", "gn_finalize+affine", "conv2")

    def __init__(self, s3dsp, ctx, cfg, torch, device, precision=None, side=None):
        self.s, self.ctx, self.torch = s3dsp, ctx, torch
        t = torch
        P = s3dsp.PREC_BF16 if precision is None else precision
        self.prec = P
        self.bf = P == s3dsp.PREC_BF16
        c = cfg["channels"]
        n = len(cfg["coords"])
        self.n, self.c = n, c
        dev = lambda a: t.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        self.coords = dev(cfg["coords"])
        self.x = dev(cfg["feats"])
        self.w1 = t.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=t.uint8, device=device)
        self.w2 = t.empty_like(self.w1)
        ctx.weights_pack(t.from_numpy(cfg["w1"]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, self.w1)
        ctx.weights_pack(t.from_numpy(cfg["w2"]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, self.w2)
        self.b1, self.b2 = dev(cfg["b1"]), dev(cfg["b2"])
        self.gamma, self.beta = dev(cfg["gamma"]), dev(cfg["beta"])
        self.part = t.empty(s3dsp.Context.gn_partials_count(n, c, 32), dtype=t.float64, device=device)
        self.sub, self.mul, self.add = (t.empty(c, device=device) for _ in range(3))
        adt = t.bfloat16 if self.bf else t.float32
        self.xb = t.empty((n, c), dtype=t.bfloat16, device=device) if self.bf else self.x
        self.y1 = t.empty((n, c), dtype=adt, device=device)
        self.hb = t.empty((n, c), dtype=adt, device=device)
        self.out = t.empty((n, c), dtype=t.float32, device=device)
        # (side context, side stream): the bf16 convert runs there, beside the tables
        self.side = side if self.bf else None
        # our kernels per step: hash init + insert, kmap, [convert], conv1, finalize, affine, conv2
        # (3xTF32: + the TF32 split of each conv's input)
        self.launches_per_step = 7 + (1 if self.bf else 0) + (2 if P == s3dsp.PREC_F32_3XTF32 else 0)
        self.conv_kernel = ctx.conv_kernel(n, 27, c, c, P)

    def step(self, marks=None):
        """One pass of the path. `marks`: 5 events recorded between the phases
        on the main stream. The hash and kernel map are freed inside the step,
        so a captured graph owns (and releases) their memory."""
        s, ctx, t = self.s, self.ctx, self.torch
        mark = (lambda i: marks[i].record()) if marks else (lambda i: None)
        mark(0)
        join = None
        if self.bf:
            if self.side is not None:
                sctx, sst = self.side
                fork = t.cuda.Event()
                fork.record()
                sst.wait_event(fork)
                with t.cuda.stream(sst):
                    sctx.convert(self.x, self.xb)
                    join = t.cuda.Event()
                    join.record(sst)
            else:
                ctx.convert(self.x, self.xb)
        h = ctx.hash_build(self.coords)
        k = ctx.kmap_subm3(h)
        if join is not None:
            t.cuda.current_stream().wait_event(join)
        mark(1)
        ctx.conv(k, 27, self.prec, self.xb, self.w1, self.b1, self.y1, self.c, gn_partials=self.part, gn_groups=32)
        mark(2)
        ctx.gn_finalize(self.part, self.n, self.c, 32, 1e-5, self.gamma, self.beta, self.sub, self.mul, self.add)
        ctx.channel_affine(self.y1, self.sub, self.mul, self.add, True, self.hb)
        mark(3)
        ctx.conv(k, 27, self.prec, self.hb, self.w2, self.b2, self.out, self.c, residual=self.x)
        mark(4)
        k.free()
        h.free()


def pairs_of(ctx, coords, torch):
    """Valid (in, out) pairs of the kernel map, counted by the library itself."""
    h = ctx.hash_build(coords)
    k = ctx.kmap_subm3(h)
    n = coords.shape[0]
    pin = torch.empty(27 * n, dtype=torch.int32, device=coords.device)
    pout = torch.empty_like(pin)
    return int(ctx.kmap_pairs(k, pin, pout)[27])


class L2Flush:
    """Write more than L2 (evicts everything a step touched), then read a
    second buffer, so the L2 holds clean lines: the next step neither hits its
    own data nor pays for the flush's write-backs."""

    def __init__(self, torch, device):
        self.t = torch
        self.w = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.r = torch.ones(L2_FLUSH_BYTES // 8, dtype=torch.float32, device=device)
        self.acc = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self):
        self.w.fill_(1.0)
        self.t.sum(self.r, dim=0, out=self.acc)


class L2WriteFlush:
    """One write of a buffer twice the size of L2: evicts everything a call
    touched. Used inside the e2e timed region, where the write-backs of the
    dirty lines it leaves are charged to the call that follows it."""

    def __init__(self, torch, device):
        self.w = torch.empty(E2E_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.w.fill_(1.0)


def time_graphs(torch, stream, path, flush, steps, warmup, n_marks):
    """Captures `path.step` twice (plain, and with events between its phases),
    replays warm-up rounds, then times `steps` plain replays (the L2 flushed
    between them, outside the events) and `steps` marked replays. Every replay
    must reproduce the eager pass's output bit for bit. Returns (device ms of
    the plain steps, per-step phase ms [steps, n_marks - 1])."""
    path.step()  # eager first pass: one-time library initialisation stays out of the graph
    stream.synchronize()
    ref_out = path.out.clone()
    marks = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_marks)]
    graph, marked = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    # thread-local capture: NCCL's watchdog thread may query events meanwhile
    with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
        path.step()
    with torch.cuda.graph(marked, stream=stream, capture_error_mode="thread_local"):
        path.step(marks)
    for _ in range(warmup):
        graph.replay()
        flush()
        marked.replay()
        flush()
    stream.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        starts[i].record(stream)
        graph.replay()
        ends[i].record(stream)
        flush()
    stream.synchronize()
    dev_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if not torch.equal(path.out, ref_out):
        raise RuntimeError("the graph-replayed step's output differs from the eager step's")
    phase_ms = []
    for i in range(steps):
        marked.replay()
        flush()
        stream.synchronize()  # the phase events are re-recorded by the next replay
        phase_ms.append([marks[j].elapsed_time(marks[j + 1]) for j in range(n_marks - 1)])
    if not torch.equal(path.out, ref_out):
        raise RuntimeError("the marked replay's output differs from the eager step's")
    del graph, marked
    return dev_ms, np.array(phase_ms)


E2E_STREAMS = 4  # contexts (each its own stream) that one host thread keeps busy in the e2e measurement


def e2e_queued(s3dsp, torch, device, main_stream, queued_call, ref_out, steps, warmup, flush):
    """Device time of `steps` host-buffer calls (rounded up to a multiple of
    E2E_STREAMS) issued by one host thread round-robin over E2E_STREAMS
    contexts, each with its own stream and pinned output: the queued entry
    point returns once its copies in, kernels and copy out are on the stream,
    so one call's PCIe copies overlap another's kernels. Each call is preceded,
    on its stream, by the L2 flush, inside the timed region. The span runs from
    one event that every stream waits on to the last stream's end event. Every
    context's last output must equal `ref_out` bit for bit. Returns (ms,
    calls timed)."""
    per = max(1, -(-steps // E2E_STREAMS))
    lanes = []
    for _ in range(E2E_STREAMS):
        st = torch.cuda.Stream(device)
        lanes.append((st, s3dsp.Context(device.index, stream=st.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS),
                      torch.empty_like(ref_out).pin_memory()))
    # warm-up: at least `warmup` rounds and two seconds of queued calls before
    # the timed region (on a freshly started box the overlapped copies run at
    # about half speed for the first seconds of such traffic)
    t_end = time.perf_counter() + 2.0
    rounds = 0
    while rounds < max(8, warmup) or time.perf_counter() < t_end:
        for st, cx, out in lanes:
            with torch.cuda.stream(st):
                flush()  # as in the timed loop (torch's per-stream workspace exists before it)
            queued_call(cx, out)
        rounds += 1
        if rounds % 8 == 0:
            for st, _, _ in lanes:
                st.synchronize()
    for st, _, _ in lanes:
        st.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    final = torch.cuda.Event(enable_timing=True)
    start.record(main_stream)
    for st, _, _ in lanes:
        st.wait_event(start)
    t_issue = time.perf_counter()
    for _ in range(per):
        for st, cx, out in lanes:
            with torch.cuda.stream(st):
                flush()
            queued_call(cx, out)
    issue_ms = (time.perf_counter() - t_issue) * 1e3
    for st, _, _ in lanes:
        ev = torch.cuda.Event()
        ev.record(st)
        main_stream.wait_event(ev)
    final.record(main_stream)
    main_stream.synchronize()
    for _, cx, out in lanes:
        cx.check()
        if not torch.equal(out, ref_out):
            raise RuntimeError("a queued host call's output differs from the synchronous call's")
    return start.elapsed_time(final), per * E2E_STREAMS, issue_ms


def e2e_piped(s3dsp, torch, device, main_stream, queued_call, ref_out, steps, warmup, flush):
    """Device time of `steps` host-buffer calls queued by one host thread on
    one context with copy streams (CONTEXT_COPY_STREAMS): a call's upload runs
    on the context's copy-in stream, its tables and block on the context's
    stream, its download on the copy-out stream, so successive calls overlap
    (the library's three staging slots). Each call is preceded on the
    context's stream by the L2 flush, inside the timed region. The span runs
    from one start event (the context forked after it) to the end of the last
    download (the context joined before the end event). Both host outputs the
    calls alternate between must equal `ref_out` bit for bit. Returns (ms,
    calls timed, host issue ms)."""
    st = torch.cuda.Stream(device)
    cx = s3dsp.Context(device.index, stream=st.cuda_stream,
                       flags=s3dsp.CONTEXT_DEFERRED_CHECKS | s3dsp.CONTEXT_COPY_STREAMS)
    outs = [torch.empty_like(ref_out).pin_memory() for _ in range(2)]

    def issue(i):
        with torch.cuda.stream(st):
            flush()
        queued_call(cx, outs[i % 2])

    # warm-up as in e2e_queued: at least `warmup` calls and two seconds of traffic
    t_end = time.perf_counter() + 2.0
    i = 0
    while i < max(8, warmup) or time.perf_counter() < t_end:
        issue(i)
        i += 1
        if i % 8 == 0:
            cx.check()
    cx.check()
    start = torch.cuda.Event(enable_timing=True)
    final = torch.cuda.Event(enable_timing=True)
    start.record(main_stream)
    st.wait_event(start)
    cx.fork()
    t_issue = time.perf_counter()
    for i in range(steps):
        issue(i)
    issue_ms = (time.perf_counter() - t_issue) * 1e3
    cx.join()
    ev = torch.cuda.Event()
    ev.record(st)
    main_stream.wait_event(ev)
    final.record(main_stream)
    main_stream.synchronize()
    cx.check()
    for o in outs:
        if not torch.equal(o, ref_out):
            raise RuntimeError("a copy-stream host call's output differs from the synchronous call's")
    cx.close()
    return start.elapsed_time(final), steps, issue_ms


def gather_rows(torch, world, values):
    """Every rank's list of floats, on every rank ([world][len])."""
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    if world == 1:
        return [values]
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [o.tolist() for o in out]


def run_ours(args, rank, world, local_rank):
    import torch
    import s3dsp
    import workloads

    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    # host threads of this rank on its GPU's NUMA node, shared with the node's other ranks
    cpus = gpu_cpus(local_rank, local_world)
    all_cpus = os.sched_getaffinity(0)
    if cpus:
        os.sched_setaffinity(0, cpus)
    n_cpus = len(os.sched_getaffinity(0))
    cfg = workloads.config2(seed=0)
    if rank > 0:
        # every rank its own object of the config-2 shape (its own features):
        # independent objects, fixed work per GPU (weak scaling)
        cfg["feats"] = workloads.normal((len(cfg["coords"]), cfg["channels"]), 1000 + rank)
    # one non-default stream for everything: the library context, torch's
    # copies and the L2 flush, and the CUDA-graph capture of a step
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    side_stream = torch.cuda.Stream(device)
    side = (s3dsp.Context(local_rank, stream=side_stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS),
            side_stream)
    path = ResBlockPath(s3dsp, ctx, cfg, torch, device, side=side)
    n, c = path.n, path.c
    flush = L2Flush(torch, device)

    # ---- device-resident steps, replayed as one CUDA graph per step ----
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    t0 = time.perf_counter()
    dev_ms, phase_ms = time_graphs(torch, stream, path, flush, args.steps, args.warmup, 5)
    wall = time.perf_counter() - t0
    conv_ms = np.concatenate([phase_ms[:, 1], phase_ms[:, 3]])
    breakdown = {name: float(v) for name, v in zip(ResBlockPath.PHASES, phase_ms.mean(0))}
    breakdown["step_with_marks"] = float(phase_ms.sum(1).mean())
    breakdown["note"] = "the bf16 convert of x runs on a side stream beside hash+kmap"

    # ---- e2e: the C-ABI block call with host buffers (H2D, tables, block, D2H, sync) ----
    coords_h = torch.from_numpy(cfg["coords"]).pin_memory()
    x_h = torch.from_numpy(cfg["feats"]).pin_memory()
    out_h = torch.empty((n, c), dtype=torch.float32).pin_memory()

    def host_call(cx, out):
        cx.res_block_gn_host(s3dsp.PREC_BF16, coords_h, x_h, path.w1, path.b1, path.gamma, path.beta, path.w2,
                             path.b2, out)

    # serial: one call at a time, the L2 flushed between calls outside the events
    e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps + args.warmup):
        j = i - args.warmup
        flush()
        if j >= 0:
            e_starts[j].record(stream)
        host_call(ctx, out_h)
        if j >= 0:
            e_ends[j].record(stream)
    stream.synchronize()
    serial_ms = sum(s.elapsed_time(e) for s, e in zip(e_starts, e_ends))
    # the copies alone: the same bytes in (coords + features) and out, one step at a time
    d_in_c = torch.empty_like(coords_h, device=device)
    d_in_x = torch.empty_like(x_h, device=device)
    d_out = torch.empty_like(out_h, device=device)
    cs, ce = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cs.record(stream)
    for _ in range(args.steps):
        d_in_c.copy_(coords_h, non_blocking=True)
        d_in_x.copy_(x_h, non_blocking=True)
        out_h.copy_(d_out, non_blocking=True)
    ce.record(stream)
    stream.synchronize()
    copy_ms = cs.elapsed_time(ce) / args.steps
    host_call(ctx, out_h)  # the reference output of the queued calls
    stream.synchronize()

    def queued_call(cx, out):
        cx.res_block_gn_host_queued(s3dsp.PREC_BF16, coords_h, x_h, path.w1, path.b1, path.gamma, path.beta,
                                    path.w2, path.b2, out)

    e2e_flush = L2WriteFlush(torch, device)
    lanes_ms, lanes_steps, lanes_issue_ms = e2e_queued(s3dsp, torch, device, stream, queued_call, out_h, args.steps,
                                                       args.warmup, e2e_flush)
    pipe_ms, pipe_steps, issue_ms = e2e_piped(s3dsp, torch, device, stream, queued_call, out_h, args.steps,
                                              args.warmup, e2e_flush)
    clocks = sampler.stop()
    h2d = coords_h.numel() * 4 + x_h.numel() * 4
    d2h = out_h.numel() * 4
    ctx.check()
    per_rank = gather_rows(torch, world, [dev_ms / args.steps, copy_ms, serial_ms / args.steps,
                                          lanes_ms / lanes_steps, float(E2E_STREAMS), float(n_cpus),
                                          lanes_issue_ms / lanes_steps, pipe_ms / pipe_steps,
                                          issue_ms / pipe_steps])

    # max over ranks
    vals = torch.tensor([dev_ms, serial_ms, pipe_ms, lanes_ms], dtype=torch.float64, device=device)
    units = torch.tensor([2.0 * n * args.steps, 2.0 * n * pipe_steps, 2.0 * n * lanes_steps], dtype=torch.float64,
                         device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(units, op=torch.distributed.ReduceOp.SUM)
    dev_ms, serial_ms, pipe_ms, lanes_ms = vals.tolist()
    total_units, pipe_units, lanes_units = units.tolist()

    line = None
    if rank == 0:
        value = total_units / (dev_ms / 1e3)
        e2e_value = pipe_units / (pipe_ms / 1e3)
        hbm, tflops, tflops_sus, peak_src = load_peaks()
        P = pairs_of(ctx, path.coords, torch)
        conv_avg_ms = float(conv_ms.mean())
        # conv1 writes bf16 (2 B); conv2 writes f32 and reads the f32 skip (4 + 4 B): their mean
        roof = conv_roofline(path.conv_kernel, n, c, P, conv_avg_ms, 3.0, 2.0, tflops, hbm, peak_src)
        roof["per_conv_ms"] = {"conv1": float(phase_ms[:, 1].mean()), "conv2": float(phase_ms[:, 3].mean())}
        line = {
            "metric": METRIC, "value": value, "value_per_gpu": value / world, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded ellipsoid shells, random-init weights)",
            "config": {"workload": "config2: 64^3 shell res block C=256 (subm conv3 -> GN32 -> SiLU -> subm conv3 -> "
                                   "+skip), hash + kmap rebuilt every step",
                       "voxels": n, "pairs": P, "channels": c, "objects_per_gpu": 1,
                       "parallelism": f"objects-dp{world}",
                       "l2": "flushed between steps (512 MiB write, then 256 MiB read of another buffer)",
                       "timing": "device steps replayed as a CUDA graph of the library calls (the breakdown and "
                                 "the roofline's conv time from a second capture with events between the phases); "
                                 "e2e = the host-buffer block entry point (host coords and features in, result out) "
                                 "per step, queued by one host thread on a context with copy streams (the "
                                 "round-robin over several contexts and the synchronous one-call-at-a-time "
                                 "figures beside it)"},
            "roofline": roof,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": pipe_ms / pipe_steps,
                    "mode": "per rank: one host thread (pinned to its GPU's NUMA node) issuing "
                            "s3dsp_res_block_gn_host_queued on one context with S3DSP_CONTEXT_COPY_STREAMS "
                            "(uploads on its copy-in stream, tables and block on its stream, downloads on its "
                            "copy-out stream: one call's upload, the next one's kernels and the previous one's "
                            "download overlap); L2 flushed on the context's stream before every call (a 256 MiB "
                            "write, inside the timed region); device-timed from one start event to the last "
                            "download's end; max over ranks. lanes_* = the same calls round-robin over "
                            f"{E2E_STREAMS} contexts of one stream each; serial_* = the synchronous "
                            "s3dsp_res_block_gn_host, one call at a time",
                    "steps": pipe_steps, "lanes_value": lanes_units / (lanes_ms / 1e3),
                    "lanes_ms_per_step": lanes_ms / lanes_steps,
                    "serial_value": total_units / (serial_ms / 1e3),
                    "serial_ms_per_step": serial_ms / args.steps,
                    "per_rank_ms": [{"rank": r, "device_step": v[0], "copies_only": v[1], "call_serial": v[2],
                                     "call_lanes": v[3], "lanes": int(v[4]), "cpus": int(v[5]),
                                     "host_issue_per_call_lanes": v[6], "call_copy_streams": v[7],
                                     "host_issue_per_call": v[8]}
                                    for r, v in enumerate(per_rank)]},
            # inside the timed regions: both graphs' replays, serial host calls, e2e calls
            "gpu_launches": path.launches_per_step * (3 * args.steps + lanes_steps + pipe_steps),
            "clocks": clocks,
            "wall_s": wall,
            "breakdown_ms": breakdown,
        }
        if world == 1:
            os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses every host core
            line["cpu_baseline"] = cpu_baseline(cfg, sample_only=True)
    del path
    if not args.no_sub:
        sub = {}
        for name, fn in (("f32", sub_f32), ("objects_5a", sub_objects), ("volume_5b", sub_volume)):
            try:
                sub[name] = fn(args, rank, world, local_rank, stream, flush)
            except Exception as e:  # a sub-record's failure is reported, not fatal to the headline
                sub[name] = {"error": repr(e)[:400]}
                if world > 1:
                    raise
        if line is not None:
            line.update(sub)
            for name in ("f32", "objects_5a", "volume_5b"):
                if isinstance(sub.get(name), dict) and "gpu_launches" in sub[name]:
                    line["gpu_launches"] += sub[name]["gpu_launches"]
    return line


# ---------------------------------------------------------------------------
# sub-record: config 2 in the reference's f32 arithmetic
# ---------------------------------------------------------------------------
def sub_f32(args, rank, world, local_rank, stream, flush):
    """The config-2 step with every activation in f32: PREC_F32_STRICT (FFMA,
    f32 accumulation: the reference's own arithmetic) and PREC_F32_3XTF32
    (the tensor cores, within the F32 gate). Same timing as the headline
    (graph replays, L2 flushed between steps)."""
    import torch
    import s3dsp
    import workloads

    device = torch.device("cuda", local_rank)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    cfg = workloads.config2(seed=0)
    if rank > 0:
        cfg["feats"] = workloads.normal((len(cfg["coords"]), cfg["channels"]), 1000 + rank)
    steps, warmup = max(1, min(args.steps, 10)), max(3, min(args.warmup, 5))
    hbm, tflops, _, peak_src = load_peaks()
    res, outs, launches = {}, {}, 0
    for name, prec in (("f32_strict", s3dsp.PREC_F32_STRICT), ("f32_3xtf32", s3dsp.PREC_F32_3XTF32)):
        path = ResBlockPath(s3dsp, ctx, cfg, torch, device, precision=prec)
        dev_ms, phase_ms = time_graphs(torch, stream, path, flush, steps, warmup, 5)
        conv_ms = float(np.concatenate([phase_ms[:, 1], phase_ms[:, 3]]).mean())
        vals = torch.tensor([dev_ms, conv_ms], dtype=torch.float64, device=device)
        if world > 1:
            torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        dev_ms, conv_ms = vals.tolist()
        outs[name] = path.out.clone()
        launches += path.launches_per_step * 2 * steps
        n, c = path.n, path.c
        P = pairs_of(ctx, path.coords, torch)
        flops = 2.0 * c * c * P
        achieved = flops / (conv_ms / 1e3) / 1e12
        if prec == s3dsp.PREC_F32_STRICT:
            peak, peak_note = FFMA_PEAK_TFLOPS, "nominal FP32 FFMA peak (148 SMs x 128 lanes x 2 x 1.965 GHz)"
        else:
            peak = tflops / 2.0 / 3.0
            peak_note = (f"3xTF32 effective peak = {peak_src} bf16_tflops / 2 (TF32 runs at half the bf16 rate) / 3 "
                         "(three MMAs per product)")
        res[name] = {"value": 2.0 * n * steps * world / (dev_ms / 1e3), "unit": UNIT,
                     "ms_per_step": dev_ms / steps, "steps": steps, "warmup": warmup, "dtype": "f32",
                     "kernel": path.conv_kernel,
                     "breakdown_ms": {k: float(v) for k, v in zip(ResBlockPath.PHASES, phase_ms.mean(0))},
                     "roofline": {"bound": "fp32" if prec == s3dsp.PREC_F32_STRICT else "tensor",
                                  "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                                  "flops_per_launch": flops, "avg_launch_ms": conv_ms, "peak_source": peak_note}}
        del path
    a, b = outs["f32_3xtf32"].double(), outs["f32_strict"].double()
    rel = float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
    ctx.check()
    if rank != 0:
        return None
    res["rel_l2_3xtf32_vs_strict"] = rel
    res["gpu_launches"] = launches
    res["note"] = ("same config-2 step as the headline with f32 activations; value = all ranks' outputs / max-rank "
                   "time; the reference arm computes in f32")
    return res


# ---------------------------------------------------------------------------
# config 5b: one large volume split in Morton slabs, NCCL halo exchange
# ---------------------------------------------------------------------------
VOLUME_RES, VOLUME_THICKNESS, VOLUME_C, VOLUME_LAYERS = 512, 4.0, 128, 8  # ~2.5M voxels
EXCHANGE_SM_RESERVES = (8, 4)  # SMs the interior conv may leave to the halo exchange's NCCL kernel


def sub_volume(args, rank, world, local_rank, stream, flush, steps=None, warmup=None):
    """Config 5b: a 512^3 ellipsoid shell (thickness 4 voxels, 2,580,824
    active voxels), C = 128, 8 bf16 subm conv layers (+SiLU), through the
    C ABI only. Every rank computes its Morton slab and halo lists
    (s3dsp_shard_plan_morton); before every layer the one-voxel halo is
    swapped by s3dsp_halo_exchange (one NCCL group of send / receive per
    peer, on a second context and stream), while the rank's interior rows
    (no halo needed) are convolved on a context that leaves
    some SMs (EXCHANGE_SM_RESERVES) to the exchange; the boundary rows' conv waits
    for the halo. Strong scaling: the volume is fixed, ranks split it.

    On-box parity: after timing, layer 0 is recomputed from features that
    every rank can generate (a seeded global tensor), through the exchange,
    with the 128-row kernel on both sides, and each rank compares its own
    rows against its own whole-volume conv, bit for bit; the mismatch counts
    are summed over ranks."""
    import torch
    import s3dsp
    import workloads

    steps = steps or max(1, min(args.steps, 5))
    warmup = warmup or max(3, min(args.warmup, 3))
    device = torch.device("cuda", local_rank)
    flags = s3dsp.CONTEXT_DEFERRED_CHECKS
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=flags)       # boundary conv
    ctx_int = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=flags)   # interior conv
    xstream = torch.cuda.Stream(device)
    ctx_x = s3dsp.Context(local_rank, stream=xstream.cuda_stream, flags=flags)    # halo exchange
    t_setup = time.perf_counter()
    coords = workloads.ellipsoid_shell_device(VOLUME_RES, 0, thickness=VOLUME_THICKNESS, device=device)
    n, c = len(coords), VOLUME_C
    plan = s3dsp.ShardPlan(coords, world, rank)
    n_own, ni, n_ghost = plan.n_own, plan.n_interior, plan.n_ghost
    rows_global = np.concatenate([plan.own, plan.ghost])
    shard_coords = torch.from_numpy(np.ascontiguousarray(coords[rows_global])).to(device)
    comm = None
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device=device)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(s3dsp.nccl_unique_id()), dtype=torch.uint8))
        torch.distributed.broadcast(uid, 0)
        comm = ctx_x.nccl_comm(world, rank, bytes(uid.cpu().numpy().tobytes()))
        ctx_int.set_sm_limit(max(1, torch.cuda.get_device_properties(local_rank).multi_processor_count
                                 - EXCHANGE_SM_RESERVES[0]))
    h = ctx.hash_build(shard_coords)
    k_int = ctx.kmap_subm3_range(h, 0, ni) if ni > 0 else None
    k_bnd = ctx.kmap_subm3_range(h, ni, n_own) if n_own > ni else None
    P = s3dsp.PREC_BF16
    ws, bs = [], []
    for i in range(VOLUME_LAYERS):
        w = torch.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=torch.uint8, device=device)
        ctx.weights_pack(torch.from_numpy(workloads.conv_weight_slat(c, c, 100 + i)), s3dsp.LAYOUT_SLAT_ROW, 27, c, c,
                         P, w)
        ws.append(w)
        bs.append(torch.from_numpy(workloads.normal((c,), 200 + i, 0.1)).to(device))
    rows = n_own + n_ghost
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    xa = torch.randn((rows, c), generator=gen, device=device).to(torch.bfloat16)
    xb = torch.zeros_like(xa)
    kernel = ctx_int.conv_kernel(max(ni, 1), 27, c, c, P)
    stream.synchronize()
    setup_s = time.perf_counter() - t_setup

    # schedule of a layer at N > 1: "overlap" runs the interior rows' conv on
    # SMs - reserve beside the exchange (reserve in EXCHANGE_SM_RESERVES);
    # "serial" runs the exchange first and the interior conv on every SM
    # (better where the exchange is short: 0.03 ms at 2 GPUs against a 5 %
    # slower conv). All are timed after the warm-up and the fastest (max over
    # ranks) is kept.
    sched = {"overlap": True, "reserve": EXCHANGE_SM_RESERVES[0]}
    n_sms = torch.cuda.get_device_properties(local_rank).multi_processor_count

    def layer(cur, nxt, li, e=None, conv_flags=0):
        ready = torch.cuda.Event()
        ready.record(stream)  # this layer's input rows are complete
        done = None
        if comm is not None:
            xstream.wait_event(ready)
            if e:
                e[3].record(xstream)
            ctx_x.halo_exchange(plan, comm, cur)
            done = torch.cuda.Event()
            done.record(xstream)
            if e:
                e[4].record(xstream)
        if e:
            e[0].record(stream)  # serial: the layer (and the interior phase) include the exchange
        if done is not None and not sched["overlap"]:
            stream.wait_event(done)
            done = None
        if k_int is not None:
            (ctx_int if sched["overlap"] else ctx).conv(k_int, 27, P, cur, ws[li], bs[li], nxt[:ni], c,
                                                        flags=s3dsp.EPI_SILU | conv_flags)
        if e:
            e[1].record(stream)
        if done is not None:
            stream.wait_event(done)
        if k_bnd is not None:
            ctx.conv(k_bnd, 27, P, cur, ws[li], bs[li], nxt[ni:n_own], c, flags=s3dsp.EPI_SILU | conv_flags)
        if e:
            e[2].record(stream)

    def step(times=None):
        cur, nxt = xa, xb
        for li in range(VOLUME_LAYERS):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if times is not None else None
            layer(cur, nxt, li, e)
            if e:
                times.append(e)
            cur, nxt = nxt, cur

    # the exchange alone (nothing else on the GPU)
    alone_ms = 0.0
    if comm is not None:
        for _ in range(3):
            ctx_x.halo_exchange(plan, comm, xa)
        xstream.synchronize()
        torch.distributed.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(xstream)
        for _ in range(20):
            ctx_x.halo_exchange(plan, comm, xa)
        a1.record(xstream)
        xstream.synchronize()
        alone_ms = a0.elapsed_time(a1) / 20
    for _ in range(warmup):
        step()
    stream.synchronize()
    xstream.synchronize()
    calib = {}
    if comm is not None:
        modes = [(True, r) for r in EXCHANGE_SM_RESERVES] + [(False, 0)]
        for mode, reserve in modes:
            sched["overlap"] = mode
            sched["reserve"] = reserve
            ctx_int.set_sm_limit(max(1, n_sms - reserve) if mode else 0)
            step()  # one untimed pass in this schedule
            stream.synchronize()
            xstream.synchronize()
            torch.distributed.barrier()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            step()
            step()
            c1.record(stream)
            stream.synchronize()
            xstream.synchronize()
            t = torch.tensor([c0.elapsed_time(c1) / 2], dtype=torch.float64, device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            calib[f"overlap, SMs - {reserve}" if mode else "serial"] = t.item()
        best = min(range(len(modes)), key=lambda i: list(calib.values())[i])
        sched["overlap"], sched["reserve"] = modes[best]
        ctx_int.set_sm_limit(max(1, n_sms - sched["reserve"]) if sched["overlap"] else 0)
        kernel = (ctx_int if sched["overlap"] else ctx).conv_kernel(max(ni, 1), 27, c, c, P)
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    per_layer = []
    for i in range(steps):
        starts[i].record(stream)
        step(per_layer)
        ends[i].record(stream)
    stream.synchronize()
    xstream.synchronize()
    clocks = sampler.stop()
    dev_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    halo_ms = float(np.mean([e[3].elapsed_time(e[4]) for e in per_layer])) if comm is not None else 0.0
    int_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in per_layer]))
    layer_ms = float(np.mean([e[0].elapsed_time(e[2]) for e in per_layer]))

    # ---- on-box parity of layer 0: sharded (with the exchange) vs whole volume ----
    g = torch.Generator(device=device).manual_seed(77)
    G = torch.randn((n, c), generator=g, device=device).to(torch.bfloat16)
    own_idx = torch.from_numpy(plan.own).to(device)
    ghost_idx = torch.from_numpy(plan.ghost).to(device)
    xs = torch.zeros((rows, c), dtype=torch.bfloat16, device=device)
    xs[:n_own] = G[own_idx]
    ys = torch.empty((rows, c), dtype=torch.bfloat16, device=device)
    layer(xs, ys, 0, conv_flags=s3dsp.CONV_TILE128)
    stream.synchronize()
    xstream.synchronize()
    ghost_ok = bool(torch.equal(xs[n_own:], G[ghost_idx]))
    hf = ctx.hash_build(torch.from_numpy(coords).to(device))
    kf = ctx.kmap_subm3(hf)
    yf = torch.empty((n, c), dtype=torch.bfloat16, device=device)
    ctx.conv(kf, 27, P, G, ws[0], bs[0], yf, c, flags=s3dsp.EPI_SILU | s3dsp.CONV_TILE128)
    mism = (ys[:n_own] != yf[own_idx]).any(dim=1).sum().to(torch.float64)
    kf.free()
    hf.free()
    del G, yf, xs, ys
    ctx.check()
    ctx_x.check()
    vals = torch.tensor([dev_ms, halo_ms, int_ms, layer_ms, alone_ms], dtype=torch.float64, device=device)
    cnt = torch.tensor([mism.item(), 0.0 if ghost_ok else 1.0, float(n_own)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(cnt, op=torch.distributed.ReduceOp.SUM)
    per_rank = gather_rows(torch, world, [float(n_own), float(ni), float(n_ghost)])
    if comm is not None:
        torch.cuda.synchronize()
        s3dsp.load().s3dsp_nccl_comm_free(comm)
    plan.free(ctx)
    dev_ms, halo_ms, int_ms, layer_ms, alone_ms = vals.tolist()
    mismatched, ghost_bad, rows_checked = cnt.tolist()
    if rank != 0:
        return None
    units = float(n) * VOLUME_LAYERS * steps
    return {
        "metric": "active-voxel outputs/s (C=128 subm conv, one volume split in Morton slabs), all GPUs",
        "value": units / (dev_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": dev_ms / steps, "scaling": "strong", "dtype": "bf16",
        "config": {"workload": f"config5b: {VOLUME_RES}^3 shell (thickness {VOLUME_THICKNESS}) {n} voxels, C={c}, "
                               f"{VOLUME_LAYERS} subm conv layers (+SiLU), Morton slabs + C-ABI NCCL halo exchange",
                   "voxels": n, "parallelism": f"morton-slabs{world}", "conv_kernel_interior": kernel,
                   "interior_conv_sms": "all" if comm is None or not sched["overlap"]
                   else f"SMs - {sched['reserve']}",
                   "schedule": "one GPU" if comm is None else
                   ("overlap: interior conv beside the exchange" if sched["overlap"]
                    else "serial: exchange, then the interior conv on every SM"),
                   "schedule_ms_per_pass": calib,
                   "rows_per_rank": [{"own": int(v[0]), "interior": int(v[1]), "ghost": int(v[2])}
                                     for v in per_rank]},
        "ms_per_layer_max_rank": {"layer": layer_ms, "interior_conv": int_ms,
                                  "halo_exchange_under_overlap": halo_ms, "halo_exchange_alone": alone_ms},
        "parity": {"check": "layer 0 from a seeded global feature tensor: sharded conv over [own | ghost] rows "
                            "after s3dsp_halo_exchange vs each rank's whole-volume conv (128-row kernel on both "
                            "sides), compared bit for bit",
                   "rows_checked": int(rows_checked), "mismatched_rows": int(mismatched),
                   "ghost_rows_exact": ghost_bad == 0, "bit_exact": mismatched == 0 and ghost_bad == 0},
        "setup_s_rank0": setup_s,
        "clocks_rank0": clocks,
        "gpu_launches": VOLUME_LAYERS * steps * ((k_int is not None) + (k_bnd is not None) +
                                                 (2 if comm is not None else 0)),
    }


def run_volume(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    stream = torch.cuda.Stream(torch.device("cuda", local_rank))
    torch.cuda.set_stream(stream)
    sampler = ClockSampler(local_rank)
    sampler.start()
    rec = sub_volume(args, rank, world, local_rank, stream, None, steps=args.steps, warmup=args.warmup)
    clocks = sampler.stop()
    if rec is None:
        return None
    rec.update({"higher_is_better": True, "vs_baseline": None,
                "data": "synthetic (seeded 512^3 ellipsoid shell, random features and weights)", "clocks": clocks})
    return rec


# ---------------------------------------------------------------------------
# config 5a: a batch of independent objects through config 4, sharded by object
# ---------------------------------------------------------------------------
OBJECTS, OBJECT_RES = 64, 64


def sub_objects(args, rank, world, local_rank, stream, flush, steps=None, warmup=None):
    """Config 5a: 64 ellipsoid shells at 64^3 (random axes, seeds 0..63), each
    through the config-4 stack (bf16). Objects are dealt to ranks largest
    first (no collective on the data path). Strong scaling: the batch is
    fixed; a step is one pass over the whole batch."""
    import torch
    import s3dsp
    import shard
    import stack
    import workloads

    steps = steps or max(1, min(args.steps, 3))
    warmup = warmup or max(3, min(args.warmup, 3))
    device = torch.device("cuda", local_rank)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    shells = [workloads.ellipsoid_shell(OBJECT_RES, i) for i in range(OBJECTS)]
    sizes = [len(s_) for s_ in shells]
    mine = shard.assign_objects(sizes, world)[rank]
    st = stack.Config4Stack(s3dsp, ctx, stack.config4_params(0), s3dsp.PREC_BF16, device)
    objs = []
    for i in mine:
        lat = workloads.normal((sizes[i], stack.LATENT), 5000 + i)
        objs.append((torch.from_numpy(shells[i]).to(device), torch.from_numpy(lat).to(device)))
    units_rank = sum(stack.units(sizes[i]) for i in mine)

    def step():
        for co, lat in objs:
            st.forward(co, lat)

    for _ in range(warmup):
        step()
    stream.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    stream.synchronize()
    clocks = sampler.stop()
    dev_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    ctx.check()
    per_rank = gather_rows(torch, world, [dev_ms / steps, float(len(mine)), float(sum(sizes[i] for i in mine)),
                                          float(units_rank), float(clocks.get("sm_mhz") or 0.0)])
    vals = torch.tensor([dev_ms], dtype=torch.float64, device=device)
    units = torch.tensor([float(units_rank) * steps], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(units, op=torch.distributed.ReduceOp.SUM)
    dev_ms = vals.item()
    total_units = units.item()
    if rank != 0:
        return None
    return {
        "metric": "active-voxel outputs/s (config-4 stack over a batch of 64 objects, sharded by object), all GPUs",
        "value": total_units / (dev_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": dev_ms / steps, "scaling": "strong", "dtype": "bf16",
        "config": {"workload": "config5a: 64 objects x config 4 (Linear 8->256, 4 GN res blocks @256, subdivide "
                               "->128 + 2 blocks, subdivide ->64 + 2 blocks, Linear ->32)",
                   "objects": OBJECTS, "voxels_total": int(sum(sizes)),
                   "parallelism": f"objects-dp{world} (largest-first assignment)",
                   "per_rank": [{"rank": r, "objects": int(v[1]), "voxels": int(v[2]), "units": int(v[3]),
                                 "ms_per_step": v[0], "sm_mhz_median": v[4]} for r, v in enumerate(per_rank)]},
        "clocks_rank0": clocks,
    }


def run_objects(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    stream = torch.cuda.Stream(torch.device("cuda", local_rank))
    torch.cuda.set_stream(stream)
    sampler = ClockSampler(local_rank)
    sampler.start()
    rec = sub_objects(args, rank, world, local_rank, stream, None, steps=args.steps, warmup=args.warmup)
    clocks = sampler.stop()
    if rec is None:
        return None
    rec.update({"higher_is_better": True, "vs_baseline": None,
                "data": "synthetic (64 seeded 64^3 ellipsoid shells with random axes, random latents and weights)",
                "clocks": clocks})
    return rec


# ---------------------------------------------------------------------------
# configs 1 and 3: single layers (F32-strict or BF16)
# ---------------------------------------------------------------------------
def run_layers(args, rank, world, local_rank):
    """Config 1: one subm conv on the 64^3 shell, C = 64 (seed 0).
    Config 3: the learned stride-2 subdivide of that shell (2x2x2 transposed
    conv 128 -> 64, one GEMM onto the child-major [Np, 8*64] layout) followed
    by one subm conv at C = 64 over the 8*Np children. Tables are built once
    (outside the timed region); a step is the layer(s) alone. Replicas only:
    at N > 1 each rank runs the same layer on its own GPU."""
    import torch
    import s3dsp
    import workloads
    import oracle

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    prec = {"f32": s3dsp.PREC_F32_STRICT, "tf32": s3dsp.PREC_F32_3XTF32, "bf16": s3dsp.PREC_BF16}[args.precision]
    xdt = torch.bfloat16 if prec == s3dsp.PREC_BF16 else torch.float32
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device)

    def pack(w, layout, kvol, cin, cout):
        dst = torch.empty(s3dsp.Context.packed_bytes(prec, kvol, cin, cout), dtype=torch.uint8, device=device)
        ctx.weights_pack(torch.from_numpy(np.ascontiguousarray(w)), layout, kvol, cin, cout, prec, dst)
        return dst

    if args.workload == "config1":
        cfg = workloads.config1(0)
        coords, n, c = cfg["coords"], len(cfg["coords"]), 64
        h = ctx.hash_build(dev(coords))
        k = ctx.kmap_subm3(h)
        w = pack(cfg["weight"], s3dsp.LAYOUT_SLAT_ROW, 27, c, c)
        b = dev(cfg["bias"])
        x = dev(cfg["feats"]).to(xdt)
        out = torch.empty((n, c), dtype=torch.float32, device=device)

        def step():
            ctx.conv(k, 27, prec, x, w, b, out, c)
        units = n
        nbr = oracle.slat_tables(coords)["conv_fine"].reshape(n, 27)
        cpu = lambda: oracle.subm_conv_slat(cfg["feats"], nbr, cfg["weight"], cfg["bias"])  # noqa: E731
        P = int(ctx.kmap_pairs(k, torch.empty(27 * n, dtype=torch.int32, device=device),
                               torch.empty(27 * n, dtype=torch.int32, device=device))[27])
        flops = 2.0 * c * c * P
        desc = f"config1: one subm conv, 64^3 shell {n} voxels, C=64 ({args.precision})"
    else:
        cfg = workloads.config3(1)
        parents, np_, cin, cout = cfg["coords"], len(cfg["coords"]), cfg["cin"], cfg["cout"]
        hp = ctx.hash_build(dev(parents), reject_duplicates=True)
        cc = torch.empty((8 * np_, 4), dtype=torch.int32, device=device)
        ks = ctx.subdivide(hp, cc)  # child coords + child submanifold map
        w_up = pack(cfg["w_up"].reshape(8 * cout, cin), s3dsp.LAYOUT_LINEAR, 1, cin, 8 * cout)
        b_up = dev(np.tile(cfg["b_up"], 8))
        w = pack(workloads.slat_to_mesh_packed(cfg["w"], cout, cout), s3dsp.LAYOUT_MESH_PACKED, 27, cout, cout)
        b = dev(cfg["b"])
        x = dev(cfg["feats"]).to(xdt)
        up = torch.empty((np_, 8 * cout), dtype=xdt, device=device)  # == [8 Np, cout] child-major
        out = torch.empty((8 * np_, cout), dtype=torch.float32, device=device)

        def step():
            ctx.conv(None, 1, prec, x, w_up, b_up, up, 8 * cout)
            ctx.conv(ks, 27, prec, up.view(8 * np_, cout), w, b, out, cout)
        units = np_ + 8 * np_
        cc_h, nb = oracle.mesh_subdivide(parents)
        wl = cfg["w_up"].reshape(8 * cout, cin)

        def cpu():
            u = oracle.linear(cfg["feats"], wl, np.tile(cfg["b_up"], 8)).reshape(8 * np_, cout)
            return oracle.subm_conv_mesh(u, nb, workloads.slat_to_mesh_packed(cfg["w"], cout, cout), cfg["b"], cout)
        P = int(ctx.kmap_pairs(ks, torch.empty(27 * 8 * np_, dtype=torch.int32, device=device),
                               torch.empty(27 * 8 * np_, dtype=torch.int32, device=device))[27])
        flops = 2.0 * cin * 8 * cout * np_ + 2.0 * cout * cout * P
        desc = (f"config3: 2x2x2 transposed subdivide {np_} -> {8 * np_} voxels (128 -> 64) + subm conv C=64 "
                f"({args.precision})")
    for _ in range(args.warmup):
        step()
        flush.fill_(1.0)
    stream.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
        flush.fill_(1.0)
    stream.synchronize()
    clocks = sampler.stop()
    dev_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    ctx.check()
    vals = torch.tensor([dev_ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    dev_ms = vals.item()
    if rank != 0:
        return None
    t0 = time.perf_counter()
    cpu()
    cpu_s = time.perf_counter() - t0
    hbm, tflops, tflops_sus, peak_src = load_peaks()
    ms = dev_ms / args.steps
    peak = tflops if prec == s3dsp.PREC_BF16 else None
    ffma_peak = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal FP32 FFMA peak (TFLOP/s), the strict F32 reference
    return {
        "metric": "active-voxel outputs/s", "value": units * world / (ms / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": args.precision,
        "data": "synthetic (seeded 64^3 ellipsoid shell, random features and weights)",
        "config": {"workload": desc, "pairs": P, "l2": "flushed between steps (512 MiB write)",
                   "parallelism": f"replicas{world}"},
        "achieved_tflops": flops / (ms / 1e3) / 1e12,
        "roofline_frac": (flops / (ms / 1e3) / 1e12) / peak if peak else None,
        "frac_of_ffma_peak": None if peak else (flops / (ms / 1e3) / 1e12) / ffma_peak,
        "cpu_baseline": {"value": units / cpu_s, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                         "sample": "the same layer(s) once through the oracle's f32 restatement"},
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# the SLat generator's sparse stages (input layer + blocks, out blocks, head)
# ---------------------------------------------------------------------------
def run_slat(args, rank, world, local_rank):
    """One sparse pass of the SLat flow generator (slat_flow_graph.cpp:278-296,
    :463-531) on the config-1 shell (64^3, seed 0): input Linear 8 -> 128,
    input_blocks.0 (128), mean-pool + input_blocks.1 (128 -> 1024 coarse),
    [transformer torso: identity, dense and out of scope], out_blocks.0
    (2048-concat -> upsample -> 128), out_blocks.1 (256-concat -> 128),
    LayerNorm + Linear 128 -> 8. Per-object tables are built once (they are
    reused by all 50 flow steps); a step is one pass with the L2 flushed
    between steps. Unit: one output voxel of one conv / linear layer.
    Replicas only at N > 1."""
    import torch
    import s3dsp
    import oracle
    import slat
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    prec = {"f32": s3dsp.PREC_F32_STRICT, "tf32": s3dsp.PREC_F32_3XTF32, "bf16": s3dsp.PREC_BF16}[args.precision]
    coords = workloads.ellipsoid_shell(64, 0)
    params, mods_h = slat.slat_params(0), slat.slat_mods(0)
    x_h = workloads.normal((len(coords), slat.IN_CH), 3)
    st = slat.SlatSparse(s3dsp, ctx, params, prec, device)
    tb = slat.SlatTablesDev(s3dsp, ctx, torch.from_numpy(coords).to(device), torch)
    mods = st.mods_to_device(mods_h)
    x = torch.from_numpy(x_h).to(device)
    flush = L2Flush(torch, device)
    out = None
    for _ in range(args.warmup):
        out = st.forward(tb, x, mods)
        flush()
    stream.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        out = st.forward(tb, x, mods)
        ends[i].record(stream)
        flush()
    stream.synchronize()
    clocks = sampler.stop()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    ctx.check()
    vals = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms = vals.item()
    if rank != 0:
        return None
    u = slat.units(tb.nf, tb.nc)
    t0 = time.perf_counter()
    exp = oracle.slat_sparse_forward(coords, x_h, params, mods_h)
    cpu_s = time.perf_counter() - t0
    got = out.double().cpu().numpy()
    rel = float(np.sqrt(((got - exp) ** 2).sum() / (exp.astype(np.float64) ** 2).sum()))
    return {
        "metric": "active-voxel outputs/s (SLat generator sparse stages, one pass)", "value": u * world / (ms / 1e3),
        "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.precision,
        "data": "synthetic (seeded 64^3 ellipsoid shell, random latent, weights and adaLN vectors)",
        "config": {"workload": "SLat sparse pass: Linear 8->128, res blocks 128 (fine), 128->1024 (coarse), "
                               "2048-concat->128 (upsampled), 256-concat->128, LayerNorm + Linear 128->8; the "
                               "transformer torso between them is the identity here",
                   "fine_voxels": tb.nf, "coarse_voxels": tb.nc, "units_per_step": u,
                   "l2": "flushed between steps (512 MiB write + 256 MiB read)",
                   "parallelism": f"replicas{world}"},
        "rel_l2_vs_oracle": rel,
        "cpu_baseline": {"value": u / cpu_s, "unit": UNIT, "cores": len(os.sched_getaffinity(0)), "kind": "port",
                         "sample": "one full pass through the oracle's f32 restatement (all host threads)"},
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# the GS decoder's Swin torso (the producer of the mesh decoder's 768-channel input)
# ---------------------------------------------------------------------------
def run_gs_torso(args, rank, world, local_rank):
    """The GS decoder (gs_decoder_graph.cpp:13-155) on the config-2
    coordinates (15,159 tokens): input Linear + APE, 12 Swin blocks (window
    attention in f32 + Linears), final LayerNorm + Linear 768 -> 448. The
    window tables and APE are built once (per object); a step is one pass,
    the L2 flushed between steps. Unit: one output row of a Linear or of the
    attention. Replicas only at N > 1."""
    import torch
    import s3dsp
    import oracle
    import gs
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    prec = {"f32": s3dsp.PREC_F32_STRICT, "tf32": s3dsp.PREC_F32_3XTF32, "bf16": s3dsp.PREC_BF16}[args.precision]
    coords = workloads.config2(seed=0)["coords"]
    n = len(coords)
    params = gs.gs_params(0)
    x_h = workloads.normal((n, gs.IN_CH), 3)
    tb = gs.GsTablesDev(s3dsp, ctx, torch.from_numpy(coords).to(device), torch)
    torso = gs.GsTorso(s3dsp, ctx, params, prec, device)
    x = torch.from_numpy(x_h).to(device)
    flush = L2Flush(torch, device)
    out = None
    for _ in range(args.warmup):
        out = torso.forward(tb, x)
        flush()
    stream.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        out = torso.forward(tb, x)
        ends[i].record(stream)
        flush()
    stream.synchronize()
    clocks = sampler.stop()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    ctx.check()
    vals = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms = vals.item()
    if rank != 0:
        return None
    # CPU: the oracle's float64 restatement with the first two blocks (a bounded sample), scaled per unit
    p2 = dict(params, blocks=params["blocks"][:2])
    t0 = time.perf_counter()
    exp2 = oracle.gs_torso_forward(coords, x_h, p2)
    cpu_s = time.perf_counter() - t0
    got2 = gs.GsTorso(s3dsp, ctx, p2, prec, device).forward(tb, x).double().cpu().numpy()
    rel = float(np.sqrt(((got2 - exp2) ** 2).sum() / (exp2 ** 2).sum()))
    u = gs.units(n)
    return {
        "metric": "token rows/s (GS decoder Swin torso, one pass)", "value": u * world / (ms / 1e3),
        "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.precision,
        "data": "synthetic (the config-2 64^3 shell's coordinates, random latent and weights)",
        "config": {"workload": "GS decoder: Linear 8->768 + APE, 12 Swin blocks (C=768, 12 heads, window 8, shifts "
                               "0/4; attention f32), LayerNorm + Linear 768->448",
                   "tokens": n, "windows": [len(w) for w in tb.windows], "units_per_step": u,
                   "l2": "flushed between steps (512 MiB write + 256 MiB read)", "parallelism": f"replicas{world}"},
        "rel_l2_vs_oracle_two_blocks": rel,
        "cpu_baseline": {"value": gs.units(n, 2) / cpu_s, "unit": "rows/s", "cores": len(os.sched_getaffinity(0)),
                         "kind": "port", "sample": "input layer + the first two blocks + head through the oracle's "
                                                   "float64 numpy restatement"},
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# the coordinate pipeline in front of the path (session.cpp argwhere, prune, downsample)
# ---------------------------------------------------------------------------
def run_coords(args, rank, world, local_rank):
    """SS occupancy -> coordinates as the reference runs it before the SLat
    stage: argwhere of the 64^3 occupancy grid, surface pruning, downsample to
    at most 42,000 rows (identity below). Input: the reference's shipped SS
    decoder occupancy fixture (69,537 occupied -> 67,783 surface voxels),
    resident on the device. A step = the three calls (each returns its count
    to the host). Unit: one input occupancy cell. Replicas only at N > 1."""
    import torch
    import s3dsp
    import oracle

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream)
    bits = np.load(os.path.join(ROOT, "tests", "golden", "ss_occ_mask.npz"))["bits"]
    grid_h = np.unpackbits(bits)[: 64 ** 3].astype(np.float32).reshape(64, 64, 64)
    grid = torch.from_numpy(grid_h).to(device)
    a = torch.empty((grid.numel(), 4), dtype=torch.int32, device=device)
    b = torch.empty_like(a)
    c = torch.empty_like(a)
    counts = []

    def step():
        n = ctx.occupancy_coords(grid, a)
        m = ctx.prune_surface(a[:n], b)
        k = ctx.downsample_coords(b[:m], c, 42000, 2, 42)
        counts[:] = [n, m, k]

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    stream.synchronize()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    vals = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms = vals.item()
    if rank != 0:
        return None
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        oc = oracle.occupancy_coords(grid_h)
        pr = oracle.prune_surface(oc)
        oracle.downsample_coords(pr, 42000, 2, 42)
    cpu_s = (time.perf_counter() - t0) / reps
    cells = grid_h.size
    return {
        "metric": "occupancy cells/s (argwhere + surface prune + downsample)", "value": cells * world / (ms / 1e3),
        "unit": "cells/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int32",
        "data": "the reference's shipped 64^3 SS occupancy fixture (tests/golden/ss_occ_mask.npz)",
        "config": {"workload": "coordinate pipeline: 64^3 occupancy -> coords -> surface prune -> downsample "
                               "(max 42,000)", "counts": counts, "parallelism": f"replicas{world}",
                   "note": "each call returns its row count to the host (a stream synchronisation per call)"},
        "cpu_baseline": {"value": cells / cpu_s, "unit": "cells/s", "cores": 1, "kind": "port",
                         "sample": "the same three steps through the oracle's single-threaded restatement"},
    }


# ---------------------------------------------------------------------------
# GS decoder Swin window tables (GsTables::build)
# ---------------------------------------------------------------------------
def run_gs_tables(args, rank, world, local_rank):
    """The GS decoder's per-object tables (sparse_ops.cpp:182-270): window
    buckets for shift (0,0,0) and (4,4,4) plus the 768-channel absolute
    position embedding, over the config-2 coordinates resident on the device.
    A step = both window tables and the embedding (each table call returns its
    bucket list to the host). Unit: one voxel. Replicas only at N > 1."""
    import torch
    import s3dsp
    import oracle
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream)
    coords_h = workloads.config2(seed=0)["coords"]
    n = len(coords_h)
    coords = torch.from_numpy(coords_h).to(device)
    bkt = [torch.empty(n, dtype=torch.int32, device=device) for _ in range(2)]
    bwd = [torch.empty(n, dtype=torch.int32, device=device) for _ in range(2)]
    ape = torch.empty((n, 768), dtype=torch.float32, device=device)
    nbk = []

    def step():
        nbk[:] = [len(ctx.gs_window_tables(coords, 4 * si, bkt[si], bwd[si])) for si in (0, 1)]
        ctx.ape(coords, ape)

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    stream.synchronize()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    vals = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms = vals.item()
    if rank != 0:
        return None
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        for si in (0, 1):
            oracle.gs_window_tables(coords_h, si)
        oracle.ape(coords_h)
    cpu_s = (time.perf_counter() - t0) / reps
    return {
        "metric": "voxels/s (GS window tables, both shifts, + APE)", "value": n * world / (ms / 1e3),
        "unit": "voxels/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int32+f32",
        "data": "synthetic: the config-2 64^3 ellipsoid shell coordinates",
        "config": {"workload": "GS decoder tables: Swin windows (8^3, shifts 0 and 4) + 768-ch APE",
                   "voxels": n, "buckets": nbk, "parallelism": f"replicas{world}",
                   "note": "each table call returns its bucket list to the host (a stream synchronisation)"},
        "cpu_baseline": {"value": n / cpu_s, "unit": "voxels/s", "cores": 1, "kind": "port",
                         "sample": "the same tables through the oracle's single-threaded restatement"},
    }


# ---------------------------------------------------------------------------
# FlexiCubes extraction (the step after the path)
# ---------------------------------------------------------------------------
def run_flexicubes(args, rank, world, local_rank):
    """extract_object_mesh (mesh_extractor.cpp:95-377) on the mesh decoder's
    256^3 output for the config-1 shell after two subdivisions (970,176 cubes,
    raw [N, 101] f32). A step = one s3dsp_flexicubes_extract (two host
    synchronisations inside) + freeing its mesh. Unit: one input cube.
    Replicas only at N > 1."""
    import torch
    import s3dsp
    import oracle
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream)
    t = np.load(os.path.join(ROOT, "tests", "golden", "flexicubes_tables.npz"))
    tab = ctx.flexicubes_tables(t["dmc"], t["num_dual"], t["check"])
    coords_h, raw_h = workloads.flexicubes_input(64, 0)
    n = len(coords_h)
    coords = torch.from_numpy(coords_h).to(device)
    raw = torch.from_numpy(raw_h).to(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    counts = {}

    def step():
        m = ctx.flexicubes(tab, raw, coords)
        counts.update(vertices=m.n_vertices, faces=m.n_faces, surface=m.n_surface, edges=m.n_edges)
        m.free()

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 255)
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    stream.synchronize()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    # end to end: host raw + coords in (pinned), mesh out (vertices, attributes, faces)
    raw_p, coords_p = torch.from_numpy(raw_h).pin_memory(), torch.from_numpy(coords_h).pin_memory()
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 5))
    d2h = 0
    e_s.record(stream)
    for _ in range(e2e_steps):
        r_d = raw_p.to(device, non_blocking=True)
        c_d = coords_p.to(device, non_blocking=True)
        m = ctx.flexicubes(tab, r_d, c_d)
        out = m.host()
        d2h = out["vertices"].nbytes + out["attrs"].nbytes + out["faces"].nbytes
        m.free()
    e_e.record(stream)
    stream.synchronize()
    e2e_ms = e_s.elapsed_time(e_e) / e2e_steps
    vals = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms = vals.tolist()
    if rank != 0:
        return None
    use_ref = oracle.ref_available()
    reps = 3
    t0 = time.perf_counter()
    for _ in range(reps):
        if use_ref:
            oracle.flexicubes(raw_h, coords_h, use_ref=True)
        else:
            oracle.flexicubes(raw_h, coords_h, dict(dmc=t["dmc"], num_dual=t["num_dual"], check=t["check"]))
    cpu_s = (time.perf_counter() - t0) / reps
    in_bytes = raw_h.nbytes + coords_h.nbytes
    out_bytes = counts["vertices"] * 36 + counts["faces"] * 12 + counts["surface"] * 8 + counts["edges"] * 8
    hbm, _, _, peak_src = load_peaks()
    achieved = (in_bytes + out_bytes) / (ms / 1e3) / 1e9
    return {
        "metric": "cubes/s (FlexiCubes extraction at 256^3)", "value": n * world / (ms / 1e3), "unit": "cubes/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: config-1 shell subdivided twice (mesh decoder row order), SDF = signed distance "
                "+ noise, other channels normal",
        "config": {"workload": "FlexiCubes extraction: raw [970176, 101] f32 at 256^3 -> dual-vertex mesh",
                   "cubes": n, **counts, "parallelism": f"replicas{world}",
                   "l2": "flushed between steps (256 MiB write)",
                   "note": "the call synchronises twice (surface/edge counts, dual-vertex count)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": None, "algorithmic_bytes": in_bytes + out_bytes, "peak_source": peak_src,
                     "scope": "whole call (all kernels and both synchronisations)"},
        "e2e": {"value": n / (e2e_ms / 1e3), "unit": "cubes/s", "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": d2h},
        "cpu_baseline": {"value": n / cpu_s, "unit": "cubes/s", "cores": 1,
                         "kind": "reference" if use_ref else "port",
                         "sample": f"{reps} full extractions through "
                                   + ("the reference's extract_object_mesh (oracle/_ref)" if use_ref
                                      else "the oracle restatement")},
    }


# ---------------------------------------------------------------------------
# CPU path (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
# ---------------------------------------------------------------------------
# CPU path (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def cpu_step(cfg, threads):
    import oracle
    coords = cfg["coords"]
    n = len(coords)
    use_ref = oracle.ref_available()
    t = oracle.slat_tables(coords, use_ref=use_ref)
    nbr = t["conv_fine"].reshape(n, 27)
    out = oracle.resblock_gn(cfg["feats"], nbr, cfg["w1"], cfg["b1"], cfg["gamma"], cfg["beta"], cfg["w2"],
                             cfg["b2"], threads=threads)
    return out, use_ref


def cpu_baseline(cfg, sample_only=False, steps=1, warmup=0):
    threads = len(os.sched_getaffinity(0)) or 1
    for _ in range(warmup):
        cpu_step(cfg, threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        _, use_ref = cpu_step(cfg, threads)
    dt = (time.perf_counter() - t0) / steps
    n = len(cfg["coords"])
    out = {"value": 2.0 * n / dt, "unit": UNIT, "cores": threads,
           "kind": "reference" if use_ref else "port",
           "sample": f"one full config-2 step ({n} voxels, 2 conv layers) per timing; tables by "
                     f"{'the reference sparse_ops.cpp' if use_ref else 'the oracle restatement'}, float ops by "
                     "the oracle's restatement of the GGML op order (f32)",
           "s_per_step": dt}
    if threads > 8:
        # the reference's parity test caps GGML at 8 threads (test_objects_mesh_decoder_parity.cpp:322)
        t0 = time.perf_counter()
        cpu_step(cfg, 8)
        out["at_8_threads"] = {"value": 2.0 * n / (time.perf_counter() - t0), "cores": 8}
    return out


def run_reference(args, rank, world):
    """The reference arm: rank 0 alone runs the reference path on all host
    cores, --warmup untimed and --steps timed full config-2 steps; the other
    ranks exit without work."""
    if rank != 0:
        return None
    import workloads
    cfg = workloads.config2(seed=0)
    cb = cpu_baseline(cfg, steps=args.steps, warmup=args.warmup)
    return {
        "metric": METRIC, "value": cb["value"], "value_per_gpu": cb["value"], "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["s_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2: 64^3 shell res block C=256 (subm conv3 -> GN32 -> SiLU -> subm conv3 -> "
                               "+skip), hash + kmap rebuilt every step",
                   "voxels": len(cfg["coords"]), "channels": cfg["channels"]},
        "impl": "reference",
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "at_8_threads") if k in cb},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# single-kernel cases for ncu captures (--profile-case)
# ---------------------------------------------------------------------------
PROFILE_CASES = {
    "conv2": "config-2 conv (C=256, 15,159 voxels), 128-row kernel",
    "conv2_pairs": "config-2 conv (C=256, 15,159 voxels), the kernel s3dsp_conv picks (split-K CTA pairs)",
    "conv2_f32": "config-2 conv (C=256, 15,159 voxels) in F32 strict (FFMA kernel)",
    "conv_sk": "256^3 shell (241,978 voxels), C=256, stream-K kernel",
    "tables": "hash + submanifold kmap of the 2.58M-voxel 512^3 shell",
    "flexicubes": "FlexiCubes extraction of 970,176 cubes at 256^3",
    "conv1_tf32": "config-1 subm conv (C=64, 15,159 voxels) in 3xTF32",
    "coords": "SS occupancy -> coords -> surface prune -> downsample (64^3 fixture)",
    "gs_tables": "GS window tables (both shifts) + APE, config-2 coordinates",
    "step2": "the config-2 step (hash, kmap, convert, conv1, GN, conv2), eager",
}


def profile_case(case, reps):
    """Warms up once, then runs the kernel(s) of `case` `reps` times on one
    stream and synchronises. Inputs are larger than L2 where the case allows
    it (conv_sk: 124 MB of bf16 features; tables: 41 MB of coordinates, 168 MB
    of table, 279 MB of map; flexicubes: 392 MB of raw features)."""
    import torch
    import s3dsp
    import workloads

    ctx = s3dsp.Context(0)
    P = s3dsp.PREC_BF16
    if case in ("conv2", "conv2_pairs", "conv_sk"):
        coords = workloads.ellipsoid_shell(256 if case == "conv_sk" else 64, 0)
        n, c = len(coords), 256
        h = ctx.hash_build(torch.from_numpy(coords).cuda())
        k = ctx.kmap_subm3(h)
        w = torch.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(workloads.kaiming_normal_slat(c, c, 2)), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, w)
        x = torch.from_numpy(workloads.normal((n, c), 1)).cuda().to(torch.bfloat16)
        b = torch.from_numpy(workloads.normal((c,), 3, 0.1)).cuda()
        out = torch.empty((n, c), device="cuda")
        flags = {"conv2": s3dsp.CONV_TILE128, "conv2_pairs": 0, "conv_sk": s3dsp.CONV_STREAM_K}[case]
        for _ in range(1 + reps):
            ctx.conv(k, 27, P, x, w, b, out, c, flags=flags)
    elif case == "conv2_f32":
        coords = workloads.ellipsoid_shell(64, 0)
        n, c = len(coords), 256
        PF = s3dsp.PREC_F32_STRICT
        k = ctx.kmap_subm3(ctx.hash_build(torch.from_numpy(coords).cuda()))
        w = torch.empty(s3dsp.Context.packed_bytes(PF, 27, c, c), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(workloads.kaiming_normal_slat(c, c, 2)), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, PF, w)
        x = torch.from_numpy(workloads.normal((n, c), 1)).cuda()
        b = torch.from_numpy(workloads.normal((c,), 3, 0.1)).cuda()
        out = torch.empty((n, c), device="cuda")
        for _ in range(1 + reps):
            ctx.conv(k, 27, PF, x, w, b, out, c)
    elif case == "step2":
        stream = torch.cuda.current_stream()
        ctx2 = s3dsp.Context(0, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
        path = ResBlockPath(s3dsp, ctx2, workloads.config2(seed=0), torch, torch.device("cuda", 0))
        for _ in range(1 + reps):
            path.step()
        ctx = ctx2
    elif case == "conv1_tf32":
        cfg = workloads.config1(0)
        coords, n, c = cfg["coords"], len(cfg["coords"]), 64
        k = ctx.kmap_subm3(ctx.hash_build(torch.from_numpy(coords).cuda()))
        P3 = s3dsp.PREC_F32_3XTF32
        w = torch.empty(s3dsp.Context.packed_bytes(P3, 27, c, c), dtype=torch.uint8, device="cuda")
        ctx.weights_pack(torch.from_numpy(cfg["weight"]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P3, w)
        x = torch.from_numpy(cfg["feats"]).cuda()
        b = torch.from_numpy(cfg["bias"]).cuda()
        out = torch.empty((n, c), device="cuda")
        for _ in range(1 + reps):
            ctx.conv(k, 27, P3, x, w, b, out, c)
    elif case == "coords":
        bits = np.load(os.path.join(ROOT, "tests", "golden", "ss_occ_mask.npz"))["bits"]
        grid = torch.from_numpy(np.unpackbits(bits)[: 64 ** 3].astype(np.float32).reshape(64, 64, 64)).cuda()
        bufs = [torch.empty((grid.numel(), 4), dtype=torch.int32, device="cuda") for _ in range(3)]
        for _ in range(1 + reps):
            m1 = ctx.occupancy_coords(grid, bufs[0])
            m2 = ctx.prune_surface(bufs[0][:m1], bufs[1])
            ctx.downsample_coords(bufs[1][:m2], bufs[2], 42000, 2, 42)
    elif case == "gs_tables":
        coords = torch.from_numpy(workloads.config2(seed=0)["coords"]).cuda()
        n = coords.shape[0]
        bkt = torch.empty(n, dtype=torch.int32, device="cuda")
        bwd = torch.empty(n, dtype=torch.int32, device="cuda")
        ape = torch.empty((n, 768), device="cuda")
        for _ in range(1 + reps):
            for si in (0, 1):
                ctx.gs_window_tables(coords, 4 * si, bkt, bwd)
            ctx.ape(coords, ape)
    elif case == "flexicubes":
        t = np.load(os.path.join(ROOT, "tests", "golden", "flexicubes_tables.npz"))
        tab = ctx.flexicubes_tables(t["dmc"], t["num_dual"], t["check"])
        coords, raw = workloads.flexicubes_input(64, 0)
        dc, dr = torch.from_numpy(coords).cuda(), torch.from_numpy(raw).cuda()
        for _ in range(1 + reps):
            ctx.flexicubes(tab, dr, dc).free()
    elif case == "tables":
        coords = workloads.ellipsoid_shell_device(512, 0, thickness=4.0)  # the config-5b volume
        d = torch.from_numpy(coords).cuda()
        for _ in range(1 + reps):
            h = ctx.hash_build(d)
            k = ctx.kmap_subm3(h)
            k.free()
            h.free()
    else:
        raise SystemExit(f"unknown profile case {case!r}; one of {sorted(PROFILE_CASES)}")
    torch.cuda.synchronize()
    ctx.check()
    print(f"{case}: ok", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config2",
                    choices=["config2", "config1", "config3", "volume", "objects", "slat", "gs_torso", "coords",
                             "gs_tables", "flexicubes"],
                    help="config2: the headline (default); volume: config 5b, one volume split across ranks; "
                         "objects: config 5a, 64 objects through config 4 sharded by object; "
                         "config1 / config3: single layers; slat: the SLat generator's sparse stages; gs_torso: the GS decoder's "
                         "Swin torso; coords: the coordinate pipeline before the path; "
                         "gs_tables: the GS decoder's Swin window tables and APE; flexicubes: the mesh extraction after "
                         "the path")
    ap.add_argument("--precision", default=None, choices=["f32", "tf32", "bf16"],
                    help="config1 / config3 (default f32), slat and gs_torso (default bf16): f32 = F32-strict FFMA, "
                         "tf32 = 3xTF32 tensor cores, bf16")
    ap.add_argument("--no-sub", action="store_true", help="config2: skip the f32 / 5a / 5b sub-records")
    ap.add_argument("--profile-case", choices=sorted(PROFILE_CASES),
                    help="run one small kernel case (for ncu) and exit: " +
                         "; ".join(f"{k}: {v}" for k, v in PROFILE_CASES.items()))
    ap.add_argument("--reps", type=int, default=3, help="--profile-case repetitions after one warm-up")
    args = ap.parse_args()
    if args.precision is None:
        args.precision = "bf16" if args.workload in ("slat", "gs_torso") else "f32"
    if args.profile_case:
        profile_case(args.profile_case, args.reps)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        if world > 1:
            import datetime
            import torch
            torch.cuda.set_device(local_rank)
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                                 device_id=torch.device("cuda", local_rank))
        runner = {"config2": run_ours, "volume": run_volume, "objects": run_objects, "slat": run_slat,
                  "gs_torso": run_gs_torso,
                  "config1": run_layers,
                  "config3": run_layers, "coords": run_coords, "gs_tables": run_gs_tables,
                  "flexicubes": run_flexicubes}[args.workload]
        line = runner(args, rank, world, local_rank)
        if world > 1:
            import torch
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
    if line is not None:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
