"""Benchmark of the sparse-convolution hot path (config 2: the residual block on a 64^3 shell at C = 256).

Workload (one "step" = one pass of the whole path over one object): the
64^3 ellipsoid-shell active set (seed 0), C = 256:
  coordinate hash -> submanifold kernel map -> subm conv3 (+ GroupNorm partial
  sums) -> GroupNorm(32) finalize -> SiLU -> subm conv3 -> + skip,
bf16 tcgen05 MMAs with f32 accumulation. Metric: active-voxel outputs/s, one
unit = one output voxel of one conv layer (2 * N per step).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): objects are independent, so each rank
runs its own object (seed = rank) with no data-path collective ("weak"
scaling); timing is the max over ranks.

`--impl reference` times the reference path on the host cores instead: the
reference's own table builder (oracle/_ref, when it was built) plus the CPU
restatement of its GGML op order, all host threads.
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

METRIC = "active-voxel outputs/s per GPU (C=256 subm conv)"
UNIT = "voxel-outputs/s"
L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2
# DRAM bytes (read + write) per launch of the config-2 conv kernel, from one ncu
# capture of `python sam3d.cpp_b200/profile_case.py conv2` (profiles/conv_tc_kernel_config2.md)
CONV_TRAFFIC_BYTES = {"conv_tc_kernel": 13.02e6}


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


# ---------------------------------------------------------------------------
# our path
# ---------------------------------------------------------------------------
class ResBlockPath:
    """Config-2 residual block through the s3dsp C-ABI (device-resident)."""

    PHASES = ("hash", "kmap", "convert", "conv1", "gn_finalize+affine", "conv2")

    def __init__(self, s3dsp, ctx, cfg, torch, device):
        self.s, self.ctx, self.torch = s3dsp, ctx, torch
        t = torch
        c = cfg["channels"]
        n = len(cfg["coords"])
        self.n, self.c = n, c
        dev = lambda a: t.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        self.coords = dev(cfg["coords"])
        self.x = dev(cfg["feats"])
        P = s3dsp.PREC_BF16
        self.w1 = t.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=t.uint8, device=device)
        self.w2 = t.empty_like(self.w1)
        ctx.weights_pack(t.from_numpy(cfg["w1"]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, self.w1)
        ctx.weights_pack(t.from_numpy(cfg["w2"]), s3dsp.LAYOUT_SLAT_ROW, 27, c, c, P, self.w2)
        self.b1, self.b2 = dev(cfg["b1"]), dev(cfg["b2"])
        self.gamma, self.beta = dev(cfg["gamma"]), dev(cfg["beta"])
        self.part = t.empty(s3dsp.Context.gn_partials_count(n, c, 32), dtype=t.float64, device=device)
        self.sub, self.mul, self.add = (t.empty(c, device=device) for _ in range(3))
        self.xb = t.empty((n, c), dtype=t.bfloat16, device=device)
        self.y1 = t.empty((n, c), dtype=t.float32, device=device)
        self.hb = t.empty((n, c), dtype=t.bfloat16, device=device)
        self.out = t.empty((n, c), dtype=t.float32, device=device)
        # our kernels per step: hash init + insert, kmap, convert, conv1, finalize, affine, conv2
        self.launches_per_step = 8
        self.conv_kernel = ctx.conv_kernel(n, 27, c, c, P)

    def step(self, marks=None):
        """One pass of the path. `marks`: 7 events recorded between the phases.
        The hash and kernel map are freed inside the step, so a captured graph
        owns (and releases) their memory."""
        s, ctx = self.s, self.ctx
        mark = (lambda i: marks[i].record()) if marks else (lambda i: None)
        mark(0)
        h = ctx.hash_build(self.coords)
        mark(1)
        k = ctx.kmap_subm3(h)
        mark(2)
        ctx.convert(self.x, self.xb)
        mark(3)
        ctx.conv(k, 27, s.PREC_BF16, self.xb, self.w1, self.b1, self.y1, self.c, gn_partials=self.part, gn_groups=32)
        mark(4)
        ctx.gn_finalize(self.part, self.n, self.c, 32, 1e-5, self.gamma, self.beta, self.sub, self.mul, self.add)
        ctx.channel_affine(self.y1, self.sub, self.mul, self.add, True, self.hb)
        mark(5)
        ctx.conv(k, 27, s.PREC_BF16, self.hb, self.w2, self.b2, self.out, self.c, residual=self.x)
        mark(6)
        k.free()
        h.free()


def pairs_of(ctx, path, torch):
    """Valid (in, out) pairs of the kernel map, counted by the library itself."""
    h = ctx.hash_build(path.coords)
    k = ctx.kmap_subm3(h)
    cap = 27 * path.n
    pin = torch.empty(cap, dtype=torch.int32, device=path.coords.device)
    pout = torch.empty_like(pin)
    return int(ctx.kmap_pairs(k, pin, pout)[27])


E2E_WORKERS = 4  # concurrent host callers in the e2e measurement


def e2e_workers(s3dsp, torch, device, main_stream, host_call, ref_out, steps, warmup):
    """Device time of `steps` host-buffer calls (rounded up to a multiple of
    E2E_WORKERS) made by E2E_WORKERS threads, each with its own context, stream
    and pinned output. Each call is preceded, on its stream, by a write of
    more than L2 and a read of another buffer (the L2 flush), inside the timed
    region. The span runs from one event that every worker stream waits on to
    the last worker's end event. Every worker's last output must equal
    `ref_out` bit for bit. Returns (ms, calls timed)."""
    per = max(1, -(-steps // E2E_WORKERS))
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    flush_rd = torch.ones(L2_FLUSH_BYTES // 8, dtype=torch.float32, device=device)
    workers = []
    for _ in range(E2E_WORKERS):
        st = torch.cuda.Stream(device)
        workers.append((st, s3dsp.Context(device.index, stream=st.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS),
                        torch.empty_like(ref_out).pin_memory(),
                        torch.empty((), dtype=torch.float32, device=device)))
    start = torch.cuda.Event(enable_timing=True)
    final = torch.cuda.Event(enable_timing=True)
    ends = [torch.cuda.Event() for _ in workers]
    ready, go = threading.Barrier(E2E_WORKERS + 1), threading.Barrier(E2E_WORKERS + 1)
    errors = []

    def body(i):
        st, cx, out, acc = workers[i]
        try:
            torch.cuda.set_device(device)
            with torch.cuda.stream(st):
                for _ in range(max(2, warmup // E2E_WORKERS)):
                    host_call(cx, out)
                st.synchronize()
                ready.wait()
                go.wait()
                st.wait_event(start)
                for _ in range(per):
                    flush.fill_(1.0)
                    torch.sum(flush_rd, dim=0, out=acc)
                    host_call(cx, out)
                ends[i].record(st)
        except Exception as e:  # surfaced after the join
            errors.append(e)
            ready.abort()
            go.abort()

    threads = [threading.Thread(target=body, args=(i,)) for i in range(E2E_WORKERS)]
    for t in threads:
        t.start()
    try:
        ready.wait()
        start.record(main_stream)
        go.wait()
    except threading.BrokenBarrierError:
        pass
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    for e in ends:
        main_stream.wait_event(e)
    final.record(main_stream)
    main_stream.synchronize()
    for _, cx, out, _ in workers:
        cx.check()
        if not torch.equal(out, ref_out):
            raise RuntimeError("a concurrent host call's output differs from the serial call's")
    return start.elapsed_time(final), per * E2E_WORKERS


def run_ours(args, rank, world, local_rank):
    import torch
    import s3dsp
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
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
    path = ResBlockPath(s3dsp, ctx, cfg, torch, device)
    n, c = path.n, path.c
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    flush_rd = torch.ones(L2_FLUSH_BYTES // 8, dtype=torch.float32, device=device)
    flush_acc = torch.empty((), dtype=torch.float32, device=device)

    def flush_l2():
        # write more than L2 (evicts everything the step touched), then read a
        # second buffer so the L2 holds clean lines: the next step neither
        # hits its own data nor pays for the flush's write-backs
        flush.fill_(1.0)
        torch.sum(flush_rd, dim=0, out=flush_acc)

    # ---- device-resident steps, replayed as one CUDA graph per step ----
    path.step()  # eager first pass: one-time library initialisation stays out of the graph
    stream.synchronize()
    ref_out = path.out.clone()  # the eager pass's output: every replay must reproduce it bit for bit
    # two captures of the same step: `graph` is timed for the value; `marked`
    # records events between the phases (for the breakdown and the conv time
    # of the roofline), which also cuts the programmatic-launch overlap
    # between the kernels at each mark
    marks = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(7)]
    graph, marked = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    # thread-local capture: NCCL's watchdog thread may query events meanwhile
    with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
        path.step()
    with torch.cuda.graph(marked, stream=stream, capture_error_mode="thread_local"):
        path.step(marks)
    for _ in range(args.warmup):
        graph.replay()
        flush_l2()
        marked.replay()
        flush_l2()
    stream.synchronize()
    if world > 1:
        torch.distributed.barrier()

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t0 = time.perf_counter()
    for i in range(args.steps):
        starts[i].record(stream)
        graph.replay()
        ends[i].record(stream)
        flush_l2()
    stream.synchronize()
    wall = time.perf_counter() - t0
    dev_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if not torch.equal(path.out, ref_out):
        raise RuntimeError("the graph-replayed step's output differs from the eager step's")
    phase_ms = []
    for i in range(args.steps):
        marked.replay()
        flush_l2()
        stream.synchronize()  # the phase events are re-recorded by the next replay
        phase_ms.append([marks[j].elapsed_time(marks[j + 1]) for j in range(6)])
    phase_ms = np.array(phase_ms)
    conv_ms = np.concatenate([phase_ms[:, 3], phase_ms[:, 5]])
    breakdown = {name: float(v) for name, v in zip(ResBlockPath.PHASES, phase_ms.mean(0))}
    breakdown["step_with_marks"] = float(phase_ms.sum(1).mean())

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
        flush_l2()
        if j >= 0:
            e_starts[j].record(stream)
        host_call(ctx, out_h)
        if j >= 0:
            e_ends[j].record(stream)
    stream.synchronize()
    serial_ms = sum(s.elapsed_time(e) for s, e in zip(e_starts, e_ends))
    # serving: E2E_WORKERS host threads, each with its own context, stream and
    # output buffer, call the same entry point concurrently, so one call's
    # copies overlap another's kernels
    pipe_ms, pipe_steps = e2e_workers(s3dsp, torch, device, stream, host_call, out_h, args.steps, args.warmup)
    clocks = sampler.stop()
    h2d = coords_h.numel() * 4 + x_h.numel() * 4
    d2h = out_h.numel() * 4
    ctx.check()

    # max over ranks
    vals = torch.tensor([dev_ms, serial_ms, pipe_ms], dtype=torch.float64, device=device)
    units = torch.tensor([2.0 * n * args.steps, 2.0 * n * pipe_steps], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(units, op=torch.distributed.ReduceOp.SUM)
    dev_ms, serial_ms, pipe_ms = vals.tolist()
    total_units, pipe_units = units.tolist()
    if rank != 0:
        del graph, marked
        return None

    value = total_units / (dev_ms / 1e3)
    e2e_value = pipe_units / (pipe_ms / 1e3)
    hbm, tflops, tflops_sus, peak_src = load_peaks()
    P = pairs_of(ctx, path, torch)
    flops = 2.0 * c * c * P  # algorithmic: valid (in, out) pairs only
    conv_avg_ms = float(conv_ms.mean())
    achieved = flops / (conv_avg_ms / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded ellipsoid shells, random-init weights)",
        "config": {"workload": "config2: 64^3 shell res block C=256 (subm conv3 -> GN32 -> SiLU -> subm conv3 -> "
                               "+skip), hash + kmap rebuilt every step",
                   "voxels": n, "pairs": P, "channels": c, "objects_per_gpu": 1, "parallelism": f"objects-dp{world}",
                   "l2": "flushed between steps (512 MiB write, then 256 MiB read of another buffer)",
                   "timing": "device steps replayed as a CUDA graph of the library calls (the breakdown and "
                             "the roofline's conv time from a second capture with events between the phases); e2e = "
                             "s3dsp_res_block_gn_host (host buffers in/out) per step, called by "
                             f"{E2E_WORKERS} concurrent host threads (serial figure beside it)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tflops, "unit": "TFLOP/s",
                     "frac": achieved / tflops, "traffic": CONV_TRAFFIC_BYTES.get(path.conv_kernel),
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                     "kernel": path.conv_kernel, "flops_per_launch": flops, "avg_launch_ms": conv_avg_ms,
                     "peak_source": f"{peak_src} bf16_tflops (burst)"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": pipe_ms / pipe_steps,
                "mode": f"{E2E_WORKERS} host threads, each its own context and stream, calling "
                        "s3dsp_res_block_gn_host concurrently; L2 flushed on the calling stream before every "
                        "call (inside the timed region); device-timed from one start event to the last call's end",
                "steps": pipe_steps, "serial_value": total_units / (serial_ms / 1e3),
                "serial_ms_per_step": serial_ms / args.steps},
        # inside the timed regions: both graphs' replays, serial host calls, worker calls
        "gpu_launches": path.launches_per_step * (3 * args.steps + pipe_steps),
        "clocks": clocks,
        "wall_s": wall,
        "breakdown_ms": breakdown,
    }
    del graph, marked
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(cfg, sample_only=True)
    return line


# ---------------------------------------------------------------------------
# config 5b: one large volume split in Morton slabs, NCCL halo exchange
# ---------------------------------------------------------------------------
VOLUME_RES, VOLUME_THICKNESS, VOLUME_C, VOLUME_LAYERS = 512, 4.0, 128, 8  # ~2.5M voxels


def run_volume(args, rank, world, local_rank):
    """Config 5b: a 512^3 ellipsoid shell (thickness 4 voxels, ~2.5M active
    voxels), C = 128, 8 bf16 subm conv layers (+SiLU). Each rank owns a
    Morton slab; before every layer the one-voxel halo is swapped with one
    all-to-all (NCCL), then the rank convolves its own rows. Strong scaling:
    the volume is fixed, ranks split it. Each rank's own rows are ordered
    interior first: the interior rows' conv runs while the halo is in flight
    (second stream), the boundary rows' conv after it lands."""
    import torch
    import s3dsp
    import shard
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    coords = workloads.ellipsoid_shell(VOLUME_RES, 0, thickness=VOLUME_THICKNESS)
    n, c = len(coords), VOLUME_C
    plan = shard.plan_halos(coords, world)[rank]
    h = ctx.hash_build(torch.from_numpy(plan.shard_coords(coords)).to(device))
    ni = plan.n_interior
    # interior rows (no halo needed) and boundary rows as two maps over [own | ghost]
    k_int = ctx.kmap_subm3_range(h, 0, ni) if ni > 0 else None
    k_bnd = ctx.kmap_subm3_range(h, ni, plan.n_own) if plan.n_own > ni else None
    P = s3dsp.PREC_BF16
    ws, bs = [], []
    for i in range(VOLUME_LAYERS):
        w = torch.empty(s3dsp.Context.packed_bytes(P, 27, c, c), dtype=torch.uint8, device=device)
        ctx.weights_pack(torch.from_numpy(workloads.conv_weight_slat(c, c, 100 + i)), s3dsp.LAYOUT_SLAT_ROW, 27, c, c,
                         P, w)
        ws.append(w)
        bs.append(torch.from_numpy(workloads.normal((c,), 200 + i, 0.1)).to(device))
    rows = plan.n_own + plan.n_ghost
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    xa = torch.randn((rows, c), generator=gen, device=device).to(torch.bfloat16)
    xb = torch.zeros_like(xa)
    kernel = ctx.conv_kernel(max(ni, plan.n_own - ni), 27, c, c, P)
    xstream = torch.cuda.Stream(device)  # the halo exchange runs beside the interior conv

    def step(times=None):
        cur, nxt = xa, xb
        for li in range(VOLUME_LAYERS):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if times is not None else None
            ready = torch.cuda.Event()
            ready.record(stream)  # this layer's input rows are complete
            done = None
            if world > 1:
                with torch.cuda.stream(xstream):
                    xstream.wait_event(ready)
                    if e:
                        e[3].record(xstream)
                    shard.exchange_halo(cur, plan)
                    done = torch.cuda.Event()
                    done.record(xstream)
                    if e:
                        e[4].record(xstream)
            if e:
                e[0].record(stream)
            if k_int is not None:
                ctx.conv(k_int, 27, P, cur, ws[li], bs[li], nxt[:ni], c, flags=s3dsp.EPI_SILU)
            if e:
                e[1].record(stream)
            if done is not None:
                stream.wait_event(done)
            if k_bnd is not None:
                ctx.conv(k_bnd, 27, P, cur, ws[li], bs[li], nxt[ni:plan.n_own], c, flags=s3dsp.EPI_SILU)
            if e:
                e[2].record(stream)
                times.append(e)
            cur, nxt = nxt, cur

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    per_layer = []
    for i in range(args.steps):
        starts[i].record(stream)
        step(per_layer)
        ends[i].record(stream)
    stream.synchronize()
    clocks = sampler.stop()
    dev_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    halo_ms = float(np.mean([e[3].elapsed_time(e[4]) for e in per_layer])) if world > 1 else 0.0
    int_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in per_layer]))
    layer_ms = float(np.mean([e[0].elapsed_time(e[2]) for e in per_layer]))
    ctx.check()
    vals = torch.tensor([dev_ms, halo_ms, int_ms, layer_ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    dev_ms, halo_ms, int_ms, layer_ms = vals.tolist()
    if rank != 0:
        return None
    units = float(n) * VOLUME_LAYERS * args.steps
    hbm, tflops, tflops_sus, peak_src = load_peaks()
    return {
        "metric": "active-voxel outputs/s (C=128 subm conv, one volume split in Morton slabs)",
        "value": units / (dev_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded 512^3 ellipsoid shell, random features and weights)",
        "config": {"workload": f"config5b: {VOLUME_RES}^3 shell (thickness {VOLUME_THICKNESS}) {n} voxels, C={c}, "
                               f"{VOLUME_LAYERS} subm conv layers, Morton slabs + NCCL halo all-to-all",
                   "voxels": n, "own_rows_rank0": plan.n_own, "interior_rows_rank0": ni,
                   "ghost_rows_rank0": plan.n_ghost,
                   "parallelism": f"morton-slabs{world}", "conv_kernel": kernel},
        "breakdown_ms_per_layer": {"halo_exchange_max_rank": halo_ms, "interior_conv_max_rank": int_ms,
                                   "layer_max_rank": layer_ms,
                                   "overlap": "the halo all-to-all runs on a second stream during the interior "
                                              "rows' conv; the boundary rows' conv waits for it"},
        "gpu_launches": VOLUME_LAYERS * args.steps * ((k_int is not None) + (k_bnd is not None) +
                                                      (1 if world > 1 else 0)),
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------
# config 5a: a batch of independent objects through config 4, sharded by object
# ---------------------------------------------------------------------------
OBJECTS, OBJECT_RES = 64, 64


def run_objects(args, rank, world, local_rank):
    """Config 5a: 64 ellipsoid shells at 64^3 (random axes, seeds 0..63), each
    through the config-4 stack (bf16). Objects are dealt to ranks largest
    first (no collective on the data path). Strong scaling: the batch is
    fixed; a step is one pass over the whole batch."""
    import torch
    import s3dsp
    import shard
    import stack
    import workloads

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    ctx = s3dsp.Context(local_rank, stream=stream.cuda_stream, flags=s3dsp.CONTEXT_DEFERRED_CHECKS)
    sizes = [len(workloads.ellipsoid_shell(OBJECT_RES, i)) for i in range(OBJECTS)]
    mine = shard.assign_objects(sizes, world)[rank]
    st = stack.Config4Stack(s3dsp, ctx, stack.config4_params(0), s3dsp.PREC_BF16, device)
    objs = []
    for i in mine:
        co = workloads.ellipsoid_shell(OBJECT_RES, i)
        lat = workloads.normal((len(co), stack.LATENT), 5000 + i)
        objs.append((torch.from_numpy(co).to(device), torch.from_numpy(lat).to(device)))
    units_rank = sum(stack.units(sizes[i]) for i in mine)

    def step():
        for co, lat in objs:
            st.forward(co, lat)

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    stream.synchronize()
    clocks = sampler.stop()
    dev_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    ctx.check()
    vals = torch.tensor([dev_ms], dtype=torch.float64, device=device)
    units = torch.tensor([float(units_rank) * args.steps], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(units, op=torch.distributed.ReduceOp.SUM)
    dev_ms = vals.item()
    total_units = units.item()
    if rank != 0:
        return None
    return {
        "metric": "active-voxel outputs/s (config-4 stack over a batch of 64 objects, sharded by object)",
        "value": total_units / (dev_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (64 seeded 64^3 ellipsoid shells with random axes, random latents and weights)",
        "config": {"workload": "config5a: 64 objects x config 4 (Linear 8->256, 4 GN res blocks @256, subdivide "
                               "->128 + 2 blocks, subdivide ->64 + 2 blocks, Linear ->32)",
                   "objects": OBJECTS, "voxels_total": int(sum(sizes)), "objects_rank0": len(mine),
                   "parallelism": f"objects-dp{world} (largest-first assignment)"},
        "clocks": clocks,
    }


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
    threads = os.cpu_count() or 1
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
    if rank != 0:
        return None
    import workloads
    cfg = workloads.config2(seed=0)
    steps = max(1, min(args.steps, 3))
    cb = cpu_baseline(cfg, steps=steps, warmup=min(args.warmup, 1))
    return {
        "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": min(args.warmup, 1), "ms_per_step": cb["s_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2: 64^3 shell res block C=256, hash/tables + block per step",
                   "voxels": len(cfg["coords"]), "channels": cfg["channels"]},
        "impl": "reference",
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "at_8_threads") if k in cb},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config2",
                    choices=["config2", "config1", "config3", "volume", "objects", "coords", "gs_tables",
                             "flexicubes"],
                    help="config2: the headline (default); volume: config 5b, one volume split across ranks; "
                         "objects: config 5a, 64 objects through config 4 sharded by object; "
                         "config1 / config3: single layers; coords: the coordinate pipeline before the path; "
                         "gs_tables: the GS decoder's Swin window tables and APE; flexicubes: the mesh extraction after "
                         "the path")
    ap.add_argument("--precision", default="f32", choices=["f32", "tf32", "bf16"],
                    help="config1 / config3 only: f32 = F32-strict FFMA, tf32 = 3xTF32 tensor cores, bf16")
    args = ap.parse_args()
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
        runner = {"config2": run_ours, "volume": run_volume, "objects": run_objects, "config1": run_layers,
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
