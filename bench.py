#!/usr/bin/env python
"""Benchmark of the Clebsch-Gordan tensor-product hot path on B200.

Default workload (``--workload conv``): the fused graph convolution that BASELINE.json's
metric names at 1/2/4/8 GPUs, with C3's irreps (1x2e (x) 1x3e -> 1x2e, per-edge weights) on
the C5 graph: 200,000 nodes uniform in a periodic cube at C3's density (side 85.5 A, 5 A
cutoff), 33,514,104 directed edges, forward + backward per step, float32.  Nodes are numbered
along a Morton curve and partitioned into contiguous receiver ranges over the ranks; the halo
rows of X (forward) and dX (backward) cross NVLink with NCCL ``all_to_all_single``, overlapped
with each rank's interior edges (strong scaling: the graph is fixed as N grows).  The metric
is directed edges per second of the whole job.

At N=1 the line also carries the batch-TP headline of BASELINE configs[1] (``tp_c2``: MACE
uvu, 24 paths, 50,000 rows, fwd+bwd) and the symmetric contraction (``sc_c5``), each with its
own roofline.  Other workloads: ``--workload c2 | c2ml | c4 | sc``.

Timing: W warm-up steps, then K steps between barriers + device syncs, CUDA events on the
launching stream, max over ranks.  The conv and C2 inputs are larger than L2 (126 MB), so no
flush is needed; a batch-TP step whose algorithmic bytes are under twice L2 (C4 at 20,000
rows) flushes L2 before every step with a 256 MB memset outside the timed events, and its
time is the sum of the steps' own event intervals.  ``e2e`` repeats the step through the public module API with pinned host buffers,
host->device copies of the inputs and device->host copies of every output inside the timed
region.  ``--impl reference`` times the CPU port of the reference's e3nn-backed path (the
reference ships no CPU implementation of its own) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "TP & conv fwd+bwd edges/sec at 1/2/4/8 B200; % of HBM/tensor roofline"
UNIT = "edges/s"
HBM_FALLBACK_GBS = 6650.0


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c2ml", "c4", "conv", "sc"], default="conv")
    ap.add_argument("--conv-nodes", type=int, default=200000)
    ap.add_argument("--conv-mode", choices=["atomic", "deterministic"], default="atomic")
    ap.add_argument("--sc-nodes", type=int, default=100000)
    ap.add_argument("--rows", type=int, default=None,
                    help="TP rows per GPU (default: the BASELINE config's batch, 50,000 for "
                         "c2/c2ml, 20,000 for c4)")
    ap.add_argument("--e2e-steps", type=int, default=6)
    ap.add_argument("--e2e-chunks", type=int, default=4,
                    help="row chunks per e2e step, one CUDA stream each (copies in both "
                         "directions overlap with each other and with the kernels)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="conv: time the eager step instead of its CUDA-graph replay")
    ap.add_argument("--no-extras", action="store_true",
                    help="at N=1, skip the extra C2 TP and symmetric-contraction lines")
    return ap.parse_args()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


L2_BYTES = 126 * 1024 * 1024  # B200 L2


def _traffic(kernel_key):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if present."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed region runs.

    NVML is polled every 10 ms from a thread (nvidia-smi's own data source, without its
    start-up delay); if NVML is unavailable, an ``nvidia-smi -lms 100`` loop is read instead.
    """

    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.samples = []  # (sm_mhz, max_mhz, reasons set)
        self.proc = None
        self.stop = threading.Event()
        self.thread = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        want = str(torch.cuda.get_device_properties(self.dev).uuid).lower()
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUUID(h)
            u = (u.decode() if isinstance(u, bytes) else u).lower()
            if u.endswith(want):
                return pynvml, h
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def _poll_nvml(self, nv, h):
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = get_reasons(h)
                rs = {n for n, b in self.REASON_BITS.items() if bits & b}
                self.samples.append((float(sm), float(mx), rs))
            except Exception:
                pass
            self.stop.wait(0.01)

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rs = {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}
                self.samples.append((float(parts[1]), float(parts[2]), rs))
            except ValueError:
                continue

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll_nvml, args=(nv, h), daemon=True)
            self.thread.start()
            while not self.samples and self.thread.is_alive():
                time.sleep(0.005)
            return self
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 5:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sms = sorted(s[0] for s in self.samples)
        reasons = set().union(*(s[2] for s in self.samples))
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": sorted(reasons), "samples": len(sms),
                "source": "nvml" if self.proc is None else "nvidia-smi"}


def _dist():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        # High-priority NCCL streams: the halo exchange's kernel is scheduled ahead of the
        # interior conv kernel that becomes ready at the same time.
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local), pg_options=opts)
    else:
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
    return world, rank, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sh_inputs(rows, lmax, seed, dtype, device):
    """Real spherical harmonics of random unit vectors, computed on the device (as a model
    computes them from edge vectors), so Y is allocated like every other device input."""
    import torch

    from openequivariance_b200.problems import real_spherical_harmonics

    gen = torch.Generator(device=device).manual_seed(seed)
    vec = torch.randn(rows, 3, device=device, dtype=torch.float64, generator=gen)
    return real_spherical_harmonics(vec, lmax).to(dtype).contiguous()


# ------------------------------------------------------------------------------ TP workload


def _workload_desc(name, problem):
    mode = problem.instructions[0].connection_mode
    shared = ", shared weights" if problem.shared_weights else ""
    return (f"{name}: batch {mode} CG tensor product fwd+bwd ({len(problem.instructions)} paths"
            f"{shared}, X={problem.irreps_in1}, Y=SH l<={problem.irreps_in2.lmax}, "
            f"L3_dim={problem.irreps_out.dim})")


def _dense_flops(problem):
    """Multiply-add FLOPs per row of the channel-mixing part of uvw paths (2 mul1 mul3 d3 per
    path), the work the tensor cores do."""
    return sum(2 * i.path_shape[0] * i.path_shape[2] * (2 * problem.irreps_out[i.i_out].ir.l + 1)
               for i in problem.instructions if i.connection_mode == "uvw")


def bench_tp(args, world, rank, local):
    import numpy as np
    import torch

    import openequivariance_b200 as oeq
    from openequivariance_b200.problems import baseline_problem

    dev = torch.device("cuda", local)
    problem = baseline_problem(args.workload)
    tp = oeq.TensorProduct(problem)
    B = args.rows or (20000 if args.workload == "c4" else 50000)
    shared = problem.shared_weights
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    X = torch.randn(B, problem.irreps_in1.dim, device=dev, generator=gen)
    Y = _sh_inputs(B, problem.irreps_in2.lmax, 99 + rank, torch.float32, dev)
    if shared:  # C4: W ~ N(0, 1/sqrt(fan_in)), fan_in = 32 channels x paths into an output
        fan = max(sum(1 for j in problem.instructions if j.i_out == i.i_out) * i.path_shape[0]
                  for i in problem.instructions)
        W = torch.randn(problem.weight_numel, device=dev, generator=gen) / fan ** 0.5
    else:
        W = torch.randn(B, problem.weight_numel, device=dev, generator=gen)
    G = torch.randn(B, problem.irreps_out.dim, device=dev, generator=gen)
    ops = torch.ops.libtorch_tp_jit

    def step():
        Z = ops.jit_tp_forward(tp.kernel, tp.hash, X, Y, W, tp.L3_dim)
        gX, gY, gW = ops.jit_tp_backward(tp.kernel, tp.hash, X, Y, W, G)
        return Z, gX, gY, gW

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches = _launches_per_step(step)
    s = 4
    d1, d2, d3, wn = (problem.irreps_in1.dim, problem.irreps_in2.dim, problem.irreps_out.dim,
                      problem.weight_numel)
    wrow = 0 if shared else wn
    bytes_fwd = B * (d1 + d2 + d3 + wrow) * s + (wn * s if shared else 0)
    bytes_bwd = B * (2 * d1 + 2 * d2 + d3 + 2 * wrow) * s + (2 * wn * s if shared else 0)
    # A step that fits in L2 would find its inputs there on the next step: flush L2 before
    # every step (outside the step's own events) and time the steps alone.
    flush = bytes_fwd + bytes_bwd < 2 * L2_BYTES
    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if flush else None
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record()
        for k in range(K):
            e = ev[k]
            if flush:
                flush_buf.zero_()
            e[0].record()
            Z = ops.jit_tp_forward(tp.kernel, tp.hash, X, Y, W, tp.L3_dim)
            e[1].record()
            e[2].record()
            ops.jit_tp_backward(tp.kernel, tp.hash, X, Y, W, G)
            e[3].record()
            # Release this step's output before the next forward allocates one: the caching
            # allocator then reuses its block instead of (in some processes) mapping a new
            # multi-GB segment while the GPU idles inside the timed forward.
            del Z
        end.record()
        torch.cuda.synchronize()
    _barrier(world)
    if flush:
        elapsed_ms = _max_over_ranks(float(sum(e[0].elapsed_time(e[3]) for e in ev)), world)
    else:
        elapsed_ms = _max_over_ranks(start.elapsed_time(end), world)
    t_fwd = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    t_bwd = float(np.mean([e[2].elapsed_time(e[3]) for e in ev]))
    peak, peak_src = _peaks()
    dom = ("tp_bwd", bytes_bwd, t_bwd) if t_bwd >= t_fwd else ("tp_fwd", bytes_fwd, t_fwd)
    achieved = dom[1] / (dom[2] * 1e-3) / 1e9
    traffic = _traffic(f"{args.workload}:{dom[0]}")
    rows_total = B * world * K
    value = rows_total / (elapsed_ms * 1e-3)

    # e2e: through the public module API with pinned host buffers.  Each step's rows are split
    # into chunks, one CUDA stream per chunk: a chunk's host-to-device copies, its forward and
    # backward, and its device-to-host copies run in order on its stream, so the copies of
    # different chunks overlap in both directions (PCIe is full duplex).  Shared weights: each
    # chunk's weight gradient is a partial sum; the step adds them on the device and reads the
    # total back once.
    E = max(1, args.e2e_steps)
    NC = max(1, min(args.e2e_chunks, B))
    hX, hY, hW, hG = (t.cpu().pin_memory() for t in (X, Y, W, G))
    outs_h = [torch.empty(B, d3).pin_memory(), torch.empty(B, d1).pin_memory(),
              torch.empty(B, d2).pin_memory(), torch.empty_like(hW).pin_memory()]
    streams = [torch.cuda.Stream(dev) for _ in range(NC)]
    cuts = [B * c // NC for c in range(NC + 1)]

    def e2e_step():
        main = torch.cuda.current_stream(dev)
        parts = []
        for c, st in enumerate(streams):
            lo, hi = cuts[c], cuts[c + 1]
            with torch.cuda.stream(st):
                x = hX[lo:hi].to(dev, non_blocking=True).requires_grad_()
                y = hY[lo:hi].to(dev, non_blocking=True).requires_grad_()
                w = (hW if shared else hW[lo:hi]).to(dev, non_blocking=True).requires_grad_()
                g = hG[lo:hi].to(dev, non_blocking=True)
                z = tp(x, y, w)
                z.backward(g)
                for h, d in zip(outs_h[:3], (z.detach(), x.grad, y.grad)):
                    h[lo:hi].copy_(d, non_blocking=True)
                if shared:
                    parts.append(w.grad)
                else:
                    outs_h[3][lo:hi].copy_(w.grad, non_blocking=True)
        if shared:
            for st in streams:
                main.wait_stream(st)
            for p in parts:
                p.record_stream(main)
            outs_h[3].copy_(torch.stack(parts).sum(0), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    _barrier(world)
    t0 = time.perf_counter()
    for _ in range(E):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = _max_over_ranks(time.perf_counter() - t0, world)
    h2d = (hX.numel() + hY.numel() + hG.numel() + hW.numel() * (NC if shared else 1)) * s
    d2h = sum(h.numel() for h in outs_h) * s
    e2e = {"value": B * world * E / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "steps": E,
           "path": f"oeq.TensorProduct forward+backward (torch op API), pinned host buffers, "
                   f"{NC} row chunks on {NC} CUDA streams per step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_tp(problem, budget_s=10.0)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": _workload_desc(args.workload, problem),
                   "rows_per_gpu": B, "global_rows": B * world,
                   "l2": ("L2 flushed before every step (256 MB memset outside the timed "
                          "events); steps timed alone" if flush
                          else "inputs larger than L2 (no flush needed)"),
                   "parallelism": f"dp{world} (independent row shards)"},
        "kernels_ms": {"tp_fwd": t_fwd, "tp_bwd": t_bwd},
        "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": peak,
                     "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "algorithmic_bytes_per_launch": dom[1],
                     "fwd_frac": bytes_fwd / (t_fwd * 1e-3) / 1e9 / peak,
                     "bwd_frac": bytes_bwd / (t_bwd * 1e-3) / 1e9 / peak},
        "e2e": e2e,
        "gpu_launches": launches * K,
        "clocks": clk.summary(),
    }
    fl = _dense_flops(problem) * B
    if fl:
        # Channel mixing of uvw paths on the tensor pipe (forward): algorithmic FLOPs and the
        # FLOPs issued by the 3xTF32 split, against TF32 = half the measured dense bf16 rate.
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                tf32 = float(json.load(f)["bf16_tflops"]) / 2
            src = "measured bf16 / 2"
        except Exception:
            tf32, src = 1590.0 / 2, "fallback bf16 / 2"
        tflops = fl / (t_fwd * 1e-3) / 1e12
        line["tensor_roofline"] = {
            "kernel": "tp_fwd", "bound": "tensor", "unit": "TFLOP/s",
            "achieved_algorithmic": tflops, "achieved_issued_3xtf32": 3 * tflops,
            "peak_tf32": tf32, "peak_source": src, "frac_issued": 3 * tflops / tf32,
            "flops_per_launch": fl}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def cpu_baseline_tp(problem, budget_s=10.0, rows=None):
    """Times the CPU port on a bounded sample of the same workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as CB
    import tp_oracle as O

    p = O.Problem(
        [(m.mul, m.ir.l, m.ir.p) for m in problem.irreps_in1],
        [(m.mul, m.ir.l, m.ir.p) for m in problem.irreps_in2],
        [(m.mul, m.ir.l, m.ir.p) for m in problem.irreps_out],
        [(i.i_in1, i.i_in2, i.i_out, i.connection_mode, True) for i in problem.instructions],
        shared_weights=problem.shared_weights)
    # Grow the batch until one call takes about a second, then repeat it until the sample
    # holds about budget_s seconds of CPU work.
    n = rows or 256
    t, threads = CB.time_tp_fwd_bwd(p, n)
    while rows is None and t < 1.0 and n < 50000:
        n *= 2
        t, threads = CB.time_tp_fwd_bwd(p, n)
    total_t, total_n = t, n
    while total_t < budget_s:
        t, threads = CB.time_tp_fwd_bwd(p, n)
        total_t += t
        total_n += n
    return {"value": total_n / total_t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{total_n} rows of the same workload ({n}-row batches), forward+backward, "
                      f"float32 torch-CPU einsums, {total_t:.1f} s"}


# ----------------------------------------------------------------------------- reference


def bench_reference_conv(args, world):
    """The conv workload's reference arm: the CPU port of the reference's e3nn-backed
    convolution (gather, per-edge tensor product, scatter-add; ``E3NNConv.forward``) on all
    host threads, each step a bounded sample of the same graph family (the C3 graph: C5's
    density and degree, 5,000 nodes, 839,872 edges, built on the CPU)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as CB
    import tp_oracle as O

    import torch

    from openequivariance_b200.graph import radius_graph

    gen = torch.Generator().manual_seed(0)
    pos = torch.rand(5000, 3, generator=gen, dtype=torch.float64) * 25.0
    rows, cols, _, _ = radius_graph(pos, 25.0, 5.0)
    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    X = torch.randn(5000, 5, generator=gen)
    G = torch.randn(5000, 5, generator=gen)
    ne = 1 << 17
    Y = torch.randn(ne, 7, generator=gen)
    W = torch.randn(ne, 1, generator=gen)
    r, c = rows[:ne], cols[:ne]
    for _ in range(args.warmup):
        CB.time_conv_fwd_bwd(p, X, Y, W, G, r, c)
    times, threads = [], None
    for _ in range(args.steps):
        t, threads = CB.time_conv_fwd_bwd(p, X, Y, W, G, r, c)
        times.append(t)
    total = sum(times)
    value = ne * args.steps / total
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": _conv_desc(args.conv_nodes, C5_EDGES.get(args.conv_nodes),
                                          args.conv_mode),
                   "edges_per_step": ne,
                   "implementation": "CPU port of the reference's e3nn-backed convolution "
                                     "(torch-CPU gather / einsum / scatter-add)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{ne} edges of the C3 graph per step, forward+backward, "
                                   f"float32"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def bench_reference(args, world, rank):
    if rank != 0:
        return None
    if args.workload == "conv":
        return bench_reference_conv(args, world)
    if args.workload == "sc":
        return {"impl": "reference", "unavailable": "no CPU port of the symmetric contraction "
                                                    "is timed; use the TP or conv workloads"}
    from openequivariance_b200.problems import baseline_problem

    problem = baseline_problem(args.workload)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as CB
    import tp_oracle as O

    p = O.Problem(
        [(m.mul, m.ir.l, m.ir.p) for m in problem.irreps_in1],
        [(m.mul, m.ir.l, m.ir.p) for m in problem.irreps_in2],
        [(m.mul, m.ir.l, m.ir.p) for m in problem.irreps_out],
        [(i.i_in1, i.i_in2, i.i_out, i.connection_mode, True) for i in problem.instructions],
        shared_weights=problem.shared_weights)
    rows = 2048
    for _ in range(args.warmup):
        CB.time_tp_fwd_bwd(p, 128)
    times = []
    threads = None
    for _ in range(args.steps):
        t, threads = CB.time_tp_fwd_bwd(p, rows)
        times.append(t)
    total = sum(times)
    value = rows * args.steps / total
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": _workload_desc(args.workload, problem),
                   "rows_per_step": rows,
                   "implementation": "CPU port of the reference's e3nn path (torch-CPU einsums)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{rows} rows per step, forward+backward, float32"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _launches_per_step(step):
    """Kernels of this library (namespace oeqb) one step launches, counted by the profiler on
    an untimed step; gpu_launches = this x K."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events()
               if e.device_type == torch.autograd.DeviceType.CUDA and "oeqb::" in e.name)


def _time_steps(step, K, world, local):
    """K steps between barriers + device syncs; (max-over-ranks elapsed ms, clock summary)."""
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record()
        for _ in range(K):
            step()
        end.record()
        torch.cuda.synchronize()
    _barrier(world)
    return _max_over_ranks(start.elapsed_time(end), world), clk.summary()


def _conv_graph(n, dev):
    """The C5 graph: n nodes uniform in a periodic cube of side 25 * (n / 5000)^(1/3) A (C3's
    density), 5 A cutoff, nodes numbered along a Morton curve, receiver-sorted edges."""
    import torch

    from openequivariance_b200.graph import morton_order, radius_graph

    box = 25.0 * (n / 5000.0) ** (1.0 / 3.0)
    gen = torch.Generator().manual_seed(0)
    pos = (torch.rand(n, 3, generator=gen, dtype=torch.float64) * box).to(dev)
    pos = pos[morton_order(pos, box)]
    rows, cols, tperm, vec = radius_graph(pos, box, 5.0)
    return rows, cols, vec


# Directed edge counts of the C5-family graphs of _conv_graph (torch.rand, seed 0), by node count.
C5_EDGES = {200000: 33509164}


def _conv_desc(n, E, mode):
    edges = f"{E} directed edges" if E is not None else "C3's edge density"
    return (f"conv: C3 irreps (1x2e x 1x3e -> 1x2e, uvu, per-edge weights) fused conv fwd+bwd "
            f"on the C5 graph: periodic radius graph, {n} nodes (Morton-numbered), {edges}, "
            f"{mode}")


def _ev_ms(fn, reps=10, warm=3):
    """Average device time of fn() on the current stream (CUDA events)."""
    import torch

    for _ in range(warm):
        fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def conv_bytes(edges, nodes, fwd, det):
    """Algorithmic bytes of one C3-irreps convolution launch (float32): each input read once,
    each output written once; per edge Y (7) and W (1) values and two int64 indices, per node
    X (5) and Z (5) values; the backward reads Y, W, X, dZ and writes dY, dW, dX (plus the
    int64 transpose permutation when deterministic)."""
    if fwd:
        return edges * ((7 + 1) * 4 + 16) + nodes * (5 + 5) * 4
    return edges * (2 * (7 + 1) * 4 + 16 + (8 if det else 0)) + nodes * (5 + 5 + 5) * 4


def bench_conv(args, world, rank, local):
    """C3 irreps on the C5 graph (200,000 nodes, 33.5 M directed edges, C3's density),
    receiver-range partitioned over the ranks with halo exchange (strong scaling)."""
    import torch
    import torch.distributed as dist

    import openequivariance_b200 as oeq
    from openequivariance_b200.distributed import PartitionedConv, ReceiverPartition
    from openequivariance_b200.problems import baseline_problem, real_spherical_harmonics

    dev = torch.device("cuda", local)
    n = args.conv_nodes
    rows, cols, vec = _conv_graph(n, dev)
    E = rows.numel()
    det = args.conv_mode == "deterministic"
    problem = baseline_problem("c1")
    conv = oeq.TensorProductConv(problem, deterministic=det)
    part = ReceiverPartition.build(rows, cols, n, world, rank)
    pc = PartitionedConv(conv, part)
    g2 = torch.Generator(device=dev).manual_seed(1)
    X = torch.randn(n, 5, device=dev, generator=g2)[part.node_lo:part.node_hi].contiguous()
    Y = real_spherical_harmonics(vec[part.edge_index], 3)[:, 9:16].float().contiguous()
    W = torch.randn(part.n_edges, 1, device=dev, generator=g2)
    G = torch.randn(part.n_own, 5, device=dev, generator=g2)
    X.requires_grad_()
    Y.requires_grad_()
    W.requires_grad_()
    del vec

    def step():
        Z = pc(X, Y, W)
        return torch.autograd.grad(Z, (X, Y, W), G)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches = _launches_per_step(step)
    # The whole step (forward, autograd backward, both NCCL exchanges and every small torch
    # op) is captured once into a CUDA graph and replayed: one launch per step instead of ~25,
    # so the ranks stay in step with each other (at 8 GPUs the eager step needs more host
    # time than device time).  Every replay runs every kernel of the step.
    graph = None
    run = step
    if not args.no_graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        _barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = step()  # noqa: F841  (outputs live in the graph's pool)
        run = graph.replay
        for _ in range(args.warmup):
            run()
        torch.cuda.synchronize()
    K = args.steps
    elapsed_ms, clocks = _time_steps(run, K, world, local)
    value = E * K / (elapsed_ms * 1e-3)

    # Per-rank breakdown (untimed diagnostic pass, CUDA events): each kernel block alone, and
    # each halo exchange alone (blocking all_to_all_single, every rank in the same order).
    nl, ni = part.n_local_nodes, part.n_interior
    Xl = torch.randn(nl, 5, device=dev)
    Gl = torch.randn(nl, 5, device=dev)
    Yd, Wd = Y.detach(), W.detach()
    gX, gY, gW = torch.empty_like(Xl), torch.empty_like(Yd), torch.empty_like(Wd)
    blocks = {"int": (slice(0, ni), part.rows_int, part.cols_int, part.tperm_int),
              "bnd": (slice(ni, part.n_edges), part.rows_bnd, part.cols_bnd, part.tperm_bnd)}
    comp = {}
    for name, (sl, r_, c_, t_) in blocks.items():
        if sl.stop > sl.start:
            comp[f"fwd_{name}"] = _ev_ms(lambda: pc.fwd(Xl, Yd[sl], Wd[sl], r_, c_, t_))
            comp[f"bwd_{name}"] = _ev_ms(lambda: pc.bwd(Xl, Yd[sl], Wd[sl], Gl, r_, c_, t_, gX,
                                                          gY[sl], gW[sl]))
        else:
            comp[f"fwd_{name}"] = comp[f"bwd_{name}"] = 0.0
    if world > 1:
        send = torch.randn(int(part.send_idx.numel()), 5, device=dev)
        halo = torch.empty(part.n_halo, 5, device=dev)
        comp["exchange_x"] = _ev_ms(lambda: dist.all_to_all_single(
            halo, send, part.recv_counts, part.send_counts))
        comp["exchange_dx"] = _ev_ms(lambda: dist.all_to_all_single(
            send, halo, part.send_counts, part.recv_counts))
    keys = sorted(comp)
    vals = torch.tensor([comp[k] for k in keys], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    breakdown = {k: float(v) for k, v in zip(keys, vals.tolist())}
    kern_ms = sum(v for k, v in breakdown.items() if not k.startswith("exchange"))
    halo_tot = torch.tensor([part.n_halo, part.n_boundary], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(halo_tot)

    # Roofline of the dominant kernel: the interior-block backward of this rank.
    t_bwd = comp["bwd_int"]
    bytes_bwd = conv_bytes(ni, nl, False, det)
    peak, peak_src = _peaks()
    achieved = bytes_bwd / (t_bwd * 1e-3) / 1e9 if t_bwd else 0.0
    t_fwd = comp["fwd_int"]
    bytes_fwd = conv_bytes(ni, nl, True, det)
    tr = _traffic(f"conv_{args.conv_mode}:conv_bwd_per_edge")
    traffic = tr * ni if tr else None

    # e2e: host buffers of this rank's inputs and outputs through the same module.  Every step
    # copies its inputs in from pinned host memory and all four outputs back out.  Steps are
    # software-pipelined over three streams: the copies in of step i + 1 and the copies out of
    # step i - 1 run while step i computes (PCIe is full duplex), with two device buffer sets
    # so that a copy never overwrites data a kernel still reads.
    hX, hY, hW, hG = (t.detach().cpu().pin_memory() for t in (X, Y, W, G))
    outs = [[torch.empty(part.n_own, 5).pin_memory(), torch.empty(part.n_own, 5).pin_memory(),
             torch.empty_like(hY).pin_memory(), torch.empty_like(hW).pin_memory()]
            for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_cmp = torch.cuda.current_stream(dev)
    dbuf = [[torch.empty(t.shape, device=dev) for t in (hX, hY, hW, hG)] for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of a set landed
    ev_used = [torch.cuda.Event() for _ in range(2)]   # compute done with a set's inputs
    ev_done = [torch.cuda.Event() for _ in range(2)]   # a set's outputs computed
    ev_out = [torch.cuda.Event() for _ in range(2)]    # a set's outputs copied out
    for e_ in ev_used + ev_out:
        e_.record(s_cmp)

    def e2e_copy_in(i):
        b = i & 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])
            for d, h in zip(dbuf[b], (hX, hY, hW, hG)):
                d.copy_(h, non_blocking=True)
            ev_in[b].record(s_in)

    def e2e_compute(i):
        b = i & 1
        s_cmp.wait_event(ev_in[b])
        s_cmp.wait_event(ev_out[b])
        x, y, w = (t.detach().requires_grad_() for t in dbuf[b][:3])
        z = pc(x, y, w)
        gx, gy, gw = torch.autograd.grad(z, (x, y, w), dbuf[b][3])
        ev_used[b].record(s_cmp)
        res = (z.detach(), gx, gy, gw)
        ev_done[b].record(s_cmp)
        return res

    def e2e_copy_out(i, res):
        b = i & 1
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[b])
            for h, d in zip(outs[b], res):
                d.record_stream(s_out)
                h.copy_(d, non_blocking=True)
            ev_out[b].record(s_out)

    def e2e_run(steps):
        e2e_copy_in(0)
        for i in range(steps):
            if i + 1 < steps:
                e2e_copy_in(i + 1)
            e2e_copy_out(i, e2e_compute(i))

    e2e_run(2)
    torch.cuda.synchronize()
    E2 = max(1, args.e2e_steps)
    _barrier(world)
    t0 = time.perf_counter()
    e2e_run(E2)
    torch.cuda.synchronize()
    e2e_s = _max_over_ranks(time.perf_counter() - t0, world)
    outs = outs[0]
    h2d = sum(t.numel() for t in (hX, hY, hW, hG)) * 4
    d2h = sum(t.numel() for t in outs) * 4
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / K, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": _conv_desc(n, E, args.conv_mode),
                   "global_edges": E, "nodes": n,
                   "parallelism": f"receiver-range partition over {world} GPU(s); halo X / dX "
                                  f"exchanged with NCCL all_to_all_single, overlapped with the "
                                  f"interior edges",
                   "halo_nodes_total": int(halo_tot[0]), "boundary_edges_total": int(halo_tot[1]),
                   "cuda_graph": graph is not None,
                   "l2": "edge arrays larger than L2 (no flush needed)"},
        "breakdown_ms_max_over_ranks": breakdown,
        "kernels_ms_per_step_max_rank": kern_ms,
        "exposed_non_kernel_ms_per_step": elapsed_ms / K - kern_ms,
        "roofline": {"bound": "hbm", "kernel": "conv_bwd (interior block, rank 0)",
                     "achieved": achieved, "peak": peak, "peak_source": peak_src, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_bytes_per_launch": bytes_bwd,
                     "fwd_frac": bytes_fwd / (t_fwd * 1e-3) / 1e9 / peak if t_fwd else None},
        "e2e": {"value": E * E2 / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": E2,
                "path": "PartitionedConv forward+backward (public module API), pinned host "
                        "buffers per rank; copies in of the next step and out of the previous "
                        "step overlap each step's compute (three streams)"},
        "gpu_launches": launches * K,
        "clocks": clocks,
    }
    line["conv_kernels"] = {
        args.conv_mode: {"fwd_ms": t_fwd, "bwd_ms": t_bwd, "fwd_frac": line["roofline"]["fwd_frac"],
                         "bwd_frac": line["roofline"]["frac"]}}
    if world == 1:
        # The other mode's kernels on the same graph (the deterministic forward writes each
        # receiver row once; its backward is two passes over per-edge records).
        other = "atomic" if det else "deterministic"
        conv2 = oeq.TensorProductConv(problem, deterministic=not det)
        ops = torch.ops.libtorch_tp_jit
        tp2 = part.tperm_int if not det else conv2.dummy_transpose_perm
        Gl2 = torch.randn(nl, 5, device=dev)

        def f2():
            return ops.jit_conv_forward(conv2.kernel, conv2.hash, Xl, Yd, Wd, 5, part.rows_int,
                                        part.cols_int, conv2.workspace_buffer, tp2)

        def b2():
            return ops.jit_conv_backward(conv2.kernel, conv2.hash, Xl, Yd, Wd, Gl2, part.rows_int,
                                         part.cols_int, conv2.workspace_buffer, tp2)

        tf2, tb2 = _ev_ms(f2), _ev_ms(b2)
        line["conv_kernels"][other] = {
            "fwd_ms": tf2, "bwd_ms": tb2,
            "fwd_frac": conv_bytes(ni, nl, True, not det) / (tf2 * 1e-3) / 1e9 / peak,
            "bwd_frac": conv_bytes(ni, nl, False, not det) / (tb2 * 1e-3) / 1e9 / peak}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_conv(rows, cols)
    del graph, run  # release the captured NCCL work before the process group goes
    return line


def cpu_baseline_conv(rows, cols, budget_s=10.0):
    """CPU port (torch-CPU scatter) of the C3 conv on a bounded sample of the edges."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as CB
    import tp_oracle as O

    import torch

    p = O.make_problem("1x2e", "1x3e", "1x2e", [(0, 0, 0, "uvu", True)])
    r, c = rows.cpu(), cols.cpu()
    nodes = int(max(r.max(), c.max())) + 1
    g = torch.Generator().manual_seed(5)
    X = torch.randn(nodes, 5, generator=g)
    G = torch.randn(nodes, 5, generator=g)

    def run(n):
        Y = torch.randn(n, 7, generator=g)
        W = torch.randn(n, 1, generator=g)
        return CB.time_conv_fwd_bwd(p, X, Y, W, G, r[:n], c[:n])

    n = 1 << 16
    while True:
        t, threads = run(n)
        if t >= 1.0 or n >= len(r):
            break
        n = min(2 * n, len(r))
    total_t, total_e = t, n
    while total_t < budget_s:
        t, threads = run(n)
        total_t += t
        total_e += n
    return {"value": total_e / total_t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{total_e} edges ({n}-edge prefixes of the same graph), forward+backward, "
                      f"float32 torch-CPU gather/scatter, {total_t:.1f} s"}


def bench_sc(args, world, rank, local):
    """C5 symmetric contraction: 128x0e+128x1o+128x2e -> 128x0e+128x1o, correlation 3,
    10 elements, 100,000 nodes per GPU, fp32 forward + backward (weak scaling)."""
    import torch

    import openequivariance_b200 as oeq

    dev = torch.device("cuda", local)
    torch.manual_seed(1234 + rank)
    n, E = args.sc_nodes, 10
    mod = oeq.SymmetricContraction("128x0e+128x1o+128x2e", "128x0e+128x1o", correlation=3,
                                   num_elements=E).to(dev)
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    x = torch.randn(n, 128, 9, device=dev, generator=g).requires_grad_()
    lab = torch.randint(0, E, (n,), device=dev, generator=g)
    y = torch.nn.functional.one_hot(lab, E).float()
    gout = torch.randn(n, 512, device=dev, generator=g)
    params = list(mod.parameters())

    def step():
        out = mod(x, y)
        torch.autograd.grad(out, [x] + params, gout)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches = _launches_per_step(step)
    K = args.steps
    elapsed_ms, clocks = _time_steps(step, K, world, local)
    # FLOP roofline of the three kernels (CUDA-core FP32; no tensor cores involved): per
    # (node, channel), M = 219 monomials of degree <= 3 in the 9 components (45 + 165 of them
    # formed with one multiply each) and 4 padded output components.
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    kt = {}
    names = ("sc_fwd_kernel", "sc_bwd_dx_kernel", "sc_bwd_dcoef_kernel")
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        for k in names:
            if k in e.name:
                kt[k] = kt.get(k, 0.0) + e.time_range.elapsed_us() / 1e3
    per_nc = {"sc_fwd_kernel": 2 * 219 * 4 + 210,
              "sc_bwd_dx_kernel": 9 * (8 + 2) + 45 * (8 + 4 + 2) + 165 * (8 + 6 + 6),
              "sc_bwd_dcoef_kernel": 2 * 219 * 4 + 210}
    props = torch.cuda.get_device_properties(dev)
    mhz = clocks.get("sm_max_mhz") or 1965.0
    fp32_peak = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12
    roof = {}
    for k, f in per_nc.items():
        if k in kt and kt[k] > 0:
            tf = f * n * 128 / (kt[k] * 1e-3) / 1e12
            roof[k] = {"ms": kt[k], "tflops": tf, "frac": tf / fp32_peak,
                       "flops_per_launch": f * n * 128}
    return {
        "metric": "symmetric contraction fwd+bwd nodes/sec", "value": n * world * K / (elapsed_ms * 1e-3),
        "unit": "nodes/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": elapsed_ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "sc: MACE symmetric contraction 128x0e+128x1o+128x2e -> "
                               "128x0e+128x1o, correlation 3, 10 elements",
                   "nodes_per_gpu": n, "parallelism": f"dp{world} (independent node shards)"},
        "gpu_launches": launches * K, "clocks": clocks,
        "roofline": {"bound": "fp32 FMA (CUDA cores)", "unit": "TFLOP/s", "peak": fp32_peak,
                     "peak_source": "nominal: SMs x 128 FP32 lanes x 2 x max SM clock",
                     "kernels": roof},
    }


def _extra(line, keys=("value", "unit", "ms_per_step", "kernels_ms", "roofline",
                       "tensor_roofline", "e2e", "cpu_baseline", "config", "metric")):
    return {k: line[k] for k in keys if k in line}


def main():
    args = _args()
    world, rank, local = _dist()
    if args.impl == "reference":
        line = bench_reference(args, world, rank)
    elif args.workload == "conv":
        line = bench_conv(args, world, rank, local)
        if world == 1 and not args.no_extras:
            # The batch-TP headline (C2) and the symmetric contraction,
            # each with its own roofline, as extra keys of the N=1 line.
            import torch

            torch.cuda.empty_cache()
            a2 = argparse.Namespace(**vars(args))
            a2.workload = "c2"
            line["tp_c2"] = _extra(bench_tp(a2, world, rank, local))
            torch.cuda.empty_cache()
            a3 = argparse.Namespace(**vars(args))
            a3.workload = "sc"
            line["sc_c5"] = _extra(bench_sc(a3, world, rank, local))
    elif args.workload == "sc":
        line = bench_sc(args, world, rank, local)
    else:
        line = bench_tp(args, world, rank, local)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
