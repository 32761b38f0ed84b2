#!/usr/bin/env python
"""Benchmark of the B200 kernel backend for TileTriton's cuTile kernels.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--no-suite]

A step is one launch of the hot-path kernel over one full BASELINE-config
batch of synthetic input already resident in HBM. The headline workload is
row-wise softmax over 4096 rows x 16384 Float32 (HBM GB/s,
algorithmic bytes = read + write, the bench/bench.jl:167 convention). The
`suite` key reports the other six kernels the same way at their BASELINE
sizes (one JSON line, one object per kernel).

Multi-GPU (torchrun, one process per GPU): by default strong scaling — the
ranks split ONE BASELINE-size job (rows, elements, output columns, batches
or tokens; `value` = the job's work / the max over ranks of CUDA-event
time), and the headline is measured a second time with every rank running a
full config of its own (`weak`). `--scaling weak` makes that the primary
number. No collective on the data path. Shards that fit in L2 get a 256 MiB
flush before every timed launch. Per-rank SM clocks and launch times are in
`per_rank`.

The stdout line is compact: the contract keys plus `suite`, one array per
workload (fields in `suite_fields`). Every figure with its description goes
to stderr as a `DETAIL {...}` line and, with `--detail PATH`, to a file.
`--result-rows` adds bench/examples.jl's `RESULT` rows before the line.

`--impl reference` times the CPU restatement of the reference's algorithm
(oracle/, OpenMP on all host cores; Julia is not available on these hosts)
on the same workload — for the softmax headline the full 4096 x 16384
config per call, inputs built once — and prints the same JSON shape.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cutile-triton_b200"))

METRIC = "softmax/layernorm HBM GB/s; f16 GEMM & FMHA TFLOPS; % of B200 roofline"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------- workloads
# name -> (description, unit, bound, algorithmic work per launch)
def _wl():
    S = 8192
    return {
        "softmax": ("softmax f32, 4096 rows x 16384 contiguous, 4*N(0,1)", "GB/s", "hbm",
                    2 * 4 * 4096 * 16384),
        "vadd": ("vadd f32, N = 2^28, U(-1,1)", "GB/s", "hbm", 3 * 4 * (1 << 28)),
        "rowsum": ("rowsum f32 131072 x 512 (Julia column-major), N(0,1)", "GB/s", "hbm",
                   4 * 131072 * 512 + 4 * 131072),
        "layernorm": ("layernorm-fwd f32, 16384 rows x 4096, eps 1e-5", "GB/s", "hbm",
                      2 * 4 * 16384 * 4096 + 2 * 4 * 4096 + 2 * 4 * 16384),
        "layernorm_bwd": ("layernorm-bwd f32, 16384 rows x 4096 (dx, dw, db)", "GB/s", "hbm",
                          3 * 4 * 16384 * 4096 + 4 * 4 * 4096 + 2 * 4 * 16384),
        "layernorm_bwd_noalloc": ("layernorm-bwd f32, 16384 rows x 4096, allocation-free entry "
                                  "point (built-in dW/dB workspace)", "GB/s", "hbm",
                                  3 * 4 * 16384 * 4096 + 4 * 4 * 4096 + 2 * 4 * 16384),
        "transpose": ("transpose f32 8192 x 8192 (extra: not a BASELINE config)", "GB/s", "hbm",
                      2 * 4 * 8192 * 8192),
        "gemm": ("f16 GEMM M=N=K=8192, f32 accumulate, f16 out", "TFLOP/s", "tensor",
                 2 * 8192 ** 3),
        "bgemm": ("f16 batched GEMM 32 x (2048 x 2048 x 2048)", "TFLOP/s", "tensor",
                  32 * 2 * 2048 ** 3),
        "fmha": ("fmha fwd f16 B8 H32 S8192 D128 non-causal", "TFLOP/s", "tensor",
                 4 * 8 * 32 * S * S * 128),
        "fmha_causal": ("fmha fwd f16 B8 H32 S8192 D128 causal", "TFLOP/s", "tensor",
                        2 * 8 * 32 * S * S * 128),
        "moe": ("fused-MoE f16 GEMM, 16384 tokens, top-2 of 8 experts, N=14336, K=4096 "
                "(extra: not a BASELINE config)", "TFLOP/s", "tensor", 2 * 16384 * 2 * 14336 * 4096),
    }


WORKLOADS = _wl()
LAUNCHES_PER_STEP = {"layernorm_bwd": 2, "layernorm_bwd_noalloc": 2, "moe": 2}  # row pass + fold; row gather + GEMM
SUITE_ORDER = ["vadd", "rowsum", "softmax", "layernorm", "layernorm_bwd", "layernorm_bwd_noalloc",
               "transpose", "gemm", "bgemm", "fmha", "fmha_causal", "moe"]
NO_E2E_CPU = {"layernorm_bwd_noalloc"}  # same work as layernorm_bwd; only the device time differs


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """Per-launch DRAM bytes (dram__bytes_read.sum + write) from the committed
    ncu summaries: lines `workload <bytes>` in profiles/traffic.txt."""
    out = {}
    p = os.path.join(ROOT, "profiles", "traffic.txt")
    if os.path.exists(p):
        for line in open(p):
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


# ---------------------------------------------------------------------------- GPU side
class Case:
    """Inputs/outputs of one workload on the device plus the launch closure.

    `part` = (rank, world) makes the case this rank's 1/world share of ONE
    BASELINE-size job (strong scaling: rows, elements, output columns,
    batches or tokens, split with shard_range); None makes it a full job of
    its own (weak scaling, every rank a full config on its own seed)."""

    # name -> (units the job splits into, alignment of a shard boundary)
    UNITS = {"softmax": (4096, 1), "vadd": (1 << 28, 1024), "rowsum": (131072, 64),
             "layernorm": (16384, 1), "layernorm_bwd": (16384, 1),
             "layernorm_bwd_noalloc": (16384, 1), "transpose": (8192, 32),
             "gemm": (8192, 256), "bgemm": (32, 1), "fmha": (8, 1), "fmha_causal": (8, 1),
             "moe": (16384, 1)}

    def __init__(self, name, dev, rank, small=False, part=None):
        import torch
        from cutile_b200 import ops
        from cutile_b200.shard import shard_range

        self.name = name
        self.run_host = None  # host-buffer call of the public API, where the library has one
        T = torch
        total, align = self.UNITS[name]
        if part is not None:
            lo, hi = shard_range(total, part[0], part[1], align)
            seed = 20261201  # one job: every rank draws its own slice of the same stream
        else:
            lo, hi = 0, total
            seed = 20261201 + 1000 * rank
        self.units, self.total_units = hi - lo, total
        u = hi - lo
        if name == "softmax":
            x = ops.fill_normal(T.empty(u, 16384, device=dev), seed, 0.0, 4.0, offset=lo * 16384)
            y = T.empty_like(x)
            self.run = lambda: ops.softmax(x, y)
            self.run_host = lambda hi_, ho: ops.softmax_host(hi_[0], ho[0], dev.index or 0)
            self.inputs, self.outputs = [x], [y]
        elif name == "vadd":
            n = (1 << 26) if small else u
            a = ops.fill_uniform(T.empty(n, device=dev), seed, offset=lo)
            b = ops.fill_uniform(T.empty(n, device=dev), seed + 1, offset=lo)
            c = T.empty_like(a)
            self.run = lambda: ops.vadd(a, b, c)
            self.run_host = lambda hi_, ho: ops.vadd_host(hi_[0], hi_[1], ho[0], dev.index or 0)
            self.inputs, self.outputs = [a, b], [c]
        elif name == "rowsum":
            # Julia u x 512, column-major: this rank's rows as a matrix of its own.
            a = ops.fill_normal(T.empty(512, u, device=dev), seed, offset=lo * 512)
            out = T.empty(u, device=dev)
            self.run = lambda: ops.rowsum(a, out)
            self.inputs, self.outputs = [a], [out]
        elif name == "layernorm":
            x = ops.fill_normal(T.empty(u, 4096, device=dev), seed, offset=lo * 4096)
            w = ops.fill_normal(T.empty(4096, device=dev), seed + 1, 1.0, 0.1)
            b = ops.fill_normal(T.empty(4096, device=dev), seed + 2, 0.0, 0.1)
            y = T.empty_like(x)
            mu = T.empty(u, device=dev)
            rs = T.empty(u, device=dev)
            self.run = lambda: ops.layernorm_fwd(x, w, b, 1e-5, y, mu, rs)
            self.run_host = lambda hi_, ho: ops.layernorm_fwd_host(
                hi_[0], hi_[1], hi_[2], 1e-5, ho[0], ho[1], ho[2], dev.index or 0)
            self.inputs, self.outputs = [x, w, b], [y, mu, rs]
        elif name in ("layernorm_bwd", "layernorm_bwd_noalloc"):
            x = ops.fill_normal(T.empty(u, 4096, device=dev), seed, offset=lo * 4096)
            dy = ops.fill_normal(T.empty(u, 4096, device=dev), seed + 3, offset=lo * 4096)
            w = ops.fill_normal(T.empty(4096, device=dev), seed + 1, 1.0, 0.1)
            b = ops.fill_normal(T.empty(4096, device=dev), seed + 2, 0.0, 0.1)
            _, mu, rs = ops.layernorm_fwd(x, w, b, 1e-5)
            dx = T.empty_like(x)
            dw = T.empty(4096, device=dev)
            db = T.empty(4096, device=dev)
            if name == "layernorm_bwd":
                groups = ops.layernorm_bwd_groups(4096, u)
                part_ws = T.empty(2 * groups * 4096, device=dev)
                self.run = lambda: ops.layernorm_bwd(x, dy, w, mu, rs, dx, dw, db, part_ws, groups)
            else:
                self.run = lambda: ops.layernorm_bwd_noalloc(x, dy, w, mu, rs, dx, dw, db)
            self.inputs, self.outputs = [x, dy, w, mu, rs], [dx, dw, db]
        elif name == "transpose":
            x = ops.fill_uniform(T.empty(u, 8192, device=dev), seed, offset=lo * 8192)
            y = T.empty(8192, u, device=dev)
            self.run = lambda: ops.transpose(x, y)
            self.inputs, self.outputs = [x], [y]
        elif name == "gemm":
            # C[:, cols] = A * B[:, cols]: this rank's output columns (Julia N).
            A = ops.fill_uniform(T.empty(8192, 8192, dtype=T.float16, device=dev), seed)
            B = ops.fill_uniform(T.empty(u, 8192, dtype=T.float16, device=dev), seed + 1,
                                 offset=lo * 8192)
            C = T.empty(u, 8192, dtype=T.float16, device=dev)
            self.run = lambda: ops.matmul(A, B, C)
            self.inputs, self.outputs = [A, B], [C]
        elif name == "bgemm":
            sz = 2048 * 2048
            A = ops.fill_uniform(T.empty(u, 2048, 2048, dtype=T.float16, device=dev), seed,
                                 offset=lo * sz)
            B = ops.fill_uniform(T.empty(u, 2048, 2048, dtype=T.float16, device=dev), seed + 1,
                                 offset=lo * sz)
            C = T.empty_like(A)
            self.run = lambda: ops.bmm(A, B, C)
            self.inputs, self.outputs = [A, B], [C]
        elif name in ("fmha", "fmha_causal"):
            shape = (1, 8, 8192, 128) if small else (u, 32, 8192, 128)
            off = lo * 32 * 8192 * 128
            q = ops.fill_normal(T.empty(shape, dtype=T.float16, device=dev), seed, offset=off)
            k = ops.fill_normal(T.empty(shape, dtype=T.float16, device=dev), seed + 1, offset=off)
            v = ops.fill_normal(T.empty(shape, dtype=T.float16, device=dev), seed + 2, offset=off)
            o = T.empty_like(q)
            causal = name == "fmha_causal"
            self.run = lambda: ops.fmha(q, k, v, 1.0 / math.sqrt(128), causal, o)
            self.inputs, self.outputs = [q, k, v], [o]
        elif name == "moe":
            M, E, topk, N, K = (4096 if small else u), 8, 2, 14336, 4096
            A = ops.fill_uniform(T.empty(M, K, dtype=T.float16, device=dev), seed, offset=lo * K)
            B = ops.fill_uniform(T.empty(E, N, K, dtype=T.float16, device=dev), seed + 1,
                                 -0.05, 0.05)
            g = T.Generator().manual_seed(seed)
            ids = T.argsort(T.rand(self.total_units, E, generator=g), dim=1)[:, :topk]
            w = T.rand(self.total_units, topk, generator=g)
            ids = ids[lo:lo + M].to(T.int32).to(dev)
            w = w[lo:lo + M].contiguous().to(dev)
            sid, eid, ntp = ops.moe_align(ids, E)
            C = T.empty(M * topk, N, dtype=T.float16, device=dev)
            self.run = lambda: ops.moe_gemm(A, B, sid, eid, ntp, topk, w, C)
            self.inputs, self.outputs = [A, B, sid, eid, ntp, w], [C]
        else:
            raise ValueError(name)

    def bytes_in(self):
        return sum(t.numel() * t.element_size() for t in self.inputs)

    def bytes_out(self):
        return sum(t.numel() * t.element_size() for t in self.outputs)

    def free(self):
        self.inputs = self.outputs = None
        self.run = None


def time_device(case, steps, warmup, dist_on, flush=None):
    """W untimed steps, then exactly K steps bracketed by barrier + synchronize,
    with per-launch CUDA events on the launching (current) stream.

    When the step's data fit in L2 (`flush` is a buffer larger than L2), the
    buffer is read before every timed launch, outside its events (a read
    leaves clean lines, so the timed kernel pays no write-backs of it), and
    the total is the sum of the launch times instead of the span.
    Returns (total_ms, mean_launch_ms), each the max over ranks."""
    import torch

    for _ in range(warmup):
        case.run()
    torch.cuda.synchronize()
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    flush_out = torch.empty(flush.shape[1:], dtype=flush.dtype, device=flush.device) \
        if flush is not None else None
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for s, e in evs:
        if flush is not None:
            torch.amax(flush, dim=0, out=flush_out)
        s.record(st)
        case.run()
        e.record(st)
    torch.cuda.synchronize()
    per = [s.elapsed_time(e) for s, e in evs]
    total = sum(per) if flush is not None else evs[0][0].elapsed_time(evs[-1][1])
    srt = sorted(per)
    stats = [total, sum(per) / len(per), srt[0], srt[len(srt) // 2]]
    case.rank_launch_ms = stats[1]
    if dist_on:
        import torch.distributed as dist
        t = torch.tensor(stats, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        stats = t.tolist()
        dist.barrier()
    case.launch_stats = {"ms_min": round(stats[2], 5), "ms_median": round(stats[3], 5),
                         "ms_mean": round(stats[1], 5)}
    return stats[0], stats[1]


def time_e2e(case, steps, dev, dist_on=False):
    """Through the public API with host buffers: per step a pinned host->device
    copy of the inputs, the kernel, and a device->host copy of the result.
    Returns (ms per step, max over ranks; H2D bytes; D2H bytes) per rank."""
    import torch

    hin = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in case.inputs]
    for h, t in zip(hin, case.inputs):
        h.copy_(t)
    hout = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in case.outputs]
    st = torch.cuda.current_stream()

    if case.run_host is not None:
        # The library's host-buffer entry point: per step it copies this step's
        # inputs in and the results out itself, chunk by chunk, overlapping
        # both directions with the kernel.
        def step():
            case.run_host(hin, hout)
    else:
        def step():
            for h, t in zip(hin, case.inputs):
                t.copy_(h, non_blocking=True)
            case.run()
            for h, t in zip(hout, case.outputs):
                h.copy_(t, non_blocking=True)

    step()
    torch.cuda.synchronize()
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(st)
    for _ in range(steps):
        step()
    e.record(st)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    if dist_on:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return ms, case.bytes_in(), case.bytes_out()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()
        t0 = time.time()
        while not self.rows and time.time() - t0 < 5:
            time.sleep(0.05)

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        load = [r for r in self.rows if (num(r[4]) or 0) > 0] or self.rows
        sm = [num(r[1]) for r in load if num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows), "samples_under_load": len(load)}


def launch_path(dev):
    """Per-launch cost of a tiny softmax (64 x 1024) through the Python C-ABI
    binding: eager (host flattening + ctypes + launch) vs the same 100
    launches captured once in a CUDA graph and replayed."""
    import torch
    from cutile_b200 import ops

    x = ops.fill_normal(torch.empty(64, 1024, device=dev), 5)
    y = torch.empty_like(x)
    for _ in range(10):
        ops.softmax(x, y)
    torch.cuda.synchronize()
    n = 2000
    t0 = time.perf_counter()
    for _ in range(n):
        ops.softmax(x, y)
    torch.cuda.synchronize()
    eager_us = (time.perf_counter() - t0) / n * 1e6
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(100):
            ops.softmax(x, y)
    g.replay()
    torch.cuda.synchronize()
    reps = 20
    t0 = time.perf_counter()
    for _ in range(reps):
        g.replay()
    torch.cuda.synchronize()
    graph_us = (time.perf_counter() - t0) / (reps * 100) * 1e6
    # A tensor-core launch (host tensor-map set-up on every eager call).
    A = ops.fill_uniform(torch.empty(256, 256, dtype=torch.float16, device=dev), 6)
    B = ops.fill_uniform(torch.empty(256, 256, dtype=torch.float16, device=dev), 7)
    C = torch.empty_like(A)
    for _ in range(10):
        ops.matmul(A, B, C)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        ops.matmul(A, B, C)
    torch.cuda.synchronize()
    gemm_us = (time.perf_counter() - t0) / n * 1e6
    return {"workload": "softmax 64 x 1024 f32 and f16 GEMM 256^3, back-to-back launches, "
                        "host wall clock",
            "eager_us_per_launch": round(eager_us, 2), "graph_us_per_launch": round(graph_us, 2),
            "gemm_eager_us_per_launch": round(gemm_us, 2)}


def roofline(name, mean_ms, peaks, peak_src, traffic, work=None):
    _, unit, bound, full = WORKLOADS[name]
    work = full if work is None else work
    if bound == "hbm":
        achieved = work / (mean_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        u = "GB/s"
    else:
        achieved = work / (mean_ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops"]
        u = "TFLOP/s"
    extra = {}
    if bound == "tensor" and "bf16_tflops_sustained" in peaks:
        # Tensor kernels timed in a loop of multi-millisecond launches run under
        # the 1 kW power cap; the sustained cuBLAS figure is measured the same way.
        extra["frac_of_sustained"] = round(achieved / peaks["bf16_tflops_sustained"], 4)
    return {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": u,
            "frac": round(achieved / peak, 4), **extra, "peak_source": f"{peak_src} ({'hbm_gbs' if bound == 'hbm' else 'bf16_tflops burst'})",
            # ncu traffic is captured on full-size launches; a rank's share scales with its units
            "traffic": (traffic[name] * work / full) if name in traffic else None,
            "algorithmic_per_launch": work}


# ---------------------------------------------------------------------------- CPU side
def cpu_workload(name):
    """The CPU restatement of `name` on inputs built once: the oracle's
    float-accumulating C/OpenMP functions (all host threads) or numpy/OpenBLAS.
    Returns (call, work per call in the workload's unit, sample description,
    threads). Softmax (the headline) is the full 4096 x 16384 config; the
    others are bounded samples of their configs."""
    import numpy as np
    from oracle import oracle as O

    threads = O.threads()
    rng = np.random.default_rng(0)
    scale = 1e9 if WORKLOADS[name][1] == "GB/s" else 1e12
    if name == "layernorm_bwd_noalloc":  # the same computation on the CPU
        name = "layernorm_bwd"

    def loop(fn, work_per_call):
        return fn, work_per_call / scale

    if name == "softmax":
        rows = 4096
        x = rng.standard_normal((rows, 16384), dtype=np.float32)
        x *= 4
        y = np.empty_like(x)
        fn, wk = loop(lambda: O.softmax_f32_into(x, y, 16384, rows), 2 * 4 * rows * 16384)
        return fn, wk, "the full 4096 x 16384 config per call", threads
    if name == "vadd":
        n = 1 << 26
        a = rng.uniform(-1, 1, n).astype(np.float32)
        b = rng.uniform(-1, 1, n).astype(np.float32)
        c = np.empty_like(a)
        fn, wk = loop(lambda: O.vadd_f32_into(a, b, c), 12 * n)
        return fn, wk, "2^26 of 2^28 elements", threads
    if name == "rowsum":
        m, n = 32768, 512
        a = rng.standard_normal((n, m)).astype(np.float32)
        out = np.empty(m, np.float32)
        fn, wk = loop(lambda: O.rowsum_f32_into(a, out, m, n, 1, m), 4 * m * n + 4 * m)
        return fn, wk, f"{m} of 131072 rows x 512 (column-major)", threads
    if name == "layernorm":
        rows, n = 2048, 4096
        x = rng.standard_normal((rows, n)).astype(np.float32)
        w = np.ones(n, np.float32)
        b = np.zeros(n, np.float32)
        y = np.empty_like(x)
        mu = np.empty(rows, np.float32)
        rs = np.empty(rows, np.float32)
        fn, wk = loop(lambda: O.layernorm_f32_into(x, w, b, y, mu, rs, n, rows, 1e-5),
                 2 * 4 * rows * n)
        return fn, wk, f"{rows} of 16384 rows x 4096", threads
    if name == "transpose":
        x = rng.uniform(-1, 1, (8192, 2048)).astype(np.float32)
        y = np.empty((2048, 8192), np.float32)
        fn, wk = loop(lambda: np.copyto(y, x.T), 2 * 4 * x.size)
        return fn, wk, (f"8192 x 2048 of 8192 x 8192 with numpy copyto(x.T) (1 thread)"), 1
    if name == "layernorm_bwd":
        rows, n = 1024, 4096
        x = rng.standard_normal((rows, n)).astype(np.float32)
        dy = rng.standard_normal((rows, n)).astype(np.float32)
        w = np.ones(n, np.float32)
        mu = x.mean(axis=1).astype(np.float32)
        rs = (1 / np.sqrt(x.var(axis=1) + 1e-5)).astype(np.float32)
        fn, wk = loop(lambda: O.layernorm_bwd(x, dy, w, mu, rs), 3 * 4 * rows * n)
        return fn, wk, (f"{rows} of 16384 rows x 4096 (oracle C/OpenMP port, double accumulation)"), threads
    if name in ("gemm", "bgemm"):
        s = 2048
        A = rng.uniform(-1, 1, (s, s)).astype(np.float32)
        B = rng.uniform(-1, 1, (s, s)).astype(np.float32)
        fn, wk = loop(lambda: A @ B, 2 * s ** 3)
        return fn, wk, (f"numpy/OpenBLAS sgemm {s}^3 on Float32 copies (Julia's Float16 mul! is "
                   f"generic code)"), threads
    if name == "moe":
        T, K, N, E, topk = 1024, 4096, 2048, 8, 2
        A = rng.uniform(-1, 1, (T, K)).astype(np.float32)
        B = rng.uniform(-1, 1, (E, N, K)).astype(np.float32)
        ids = np.stack([rng.choice(E, topk, replace=False) for _ in range(T)])
        groups = [np.nonzero((ids == e).any(axis=1))[0] for e in range(E)]

        def one():
            for e in range(E):
                A[groups[e]] @ B[e].T

        fn, wk = loop(one, 2 * T * topk * N * K)
        return fn, wk, (f"{T} tokens, top-{topk} of {E} experts, N={N} of 14336, K={K}: per-expert "
                   f"gather + numpy/OpenBLAS sgemm"), threads
    if name in ("fmha", "fmha_causal"):
        S, D = 2048, 128
        q = rng.standard_normal((S, D)).astype(np.float32)
        k = rng.standard_normal((S, D)).astype(np.float32)
        vv = rng.standard_normal((S, D)).astype(np.float32)
        causal = name == "fmha_causal"
        mask = np.triu(np.ones((S, S), bool), 1) if causal else None

        def one():
            s_ = (q @ k.T) * (1 / math.sqrt(D))
            if causal:
                s_[mask] = -np.inf
            s_ -= s_.max(axis=1, keepdims=True)
            p = np.exp(s_)
            p /= p.sum(axis=1, keepdims=True)
            return p @ vv

        flops = 4 * S * S * D // (2 if causal else 1)
        fn, wk = loop(one, flops)
        return fn, wk, (f"one (batch, head) at S={S}, D={D} with numpy/OpenBLAS float32 "
                   f"(per-head mul! + softmax)"), threads
    raise ValueError(name)


def cpu_bench(name, budget_s, steps=1, warmup=1, work=None):
    """Times `name`'s CPU restatement (inputs built once, outside the timing):
    `warmup` untimed calls, then `steps` timed steps of equal call counts that
    together fill about `budget_s` seconds. value = work per call / median
    call time (robust to other processes on the host); `best` uses the
    fastest step (the min-time rule of bench/examples.jl:43-51)."""
    fn, wk, sample, threads = work or cpu_workload(name)
    for _ in range(max(1, warmup)):
        fn()
    t0 = time.perf_counter()
    fn()
    one = max(time.perf_counter() - t0, 1e-6)
    calls = max(1, int(budget_s / steps / one))
    per_call, step_ms = [], []
    for _ in range(steps):
        t0 = time.perf_counter()
        for _ in range(calls):
            t1 = time.perf_counter()
            fn()
            per_call.append(time.perf_counter() - t1)
        step_ms.append((time.perf_counter() - t0) * 1e3)
    med = statistics.median(per_call)
    return {"value": wk / med, "best": wk / min(per_call), "mean": wk * len(per_call) / sum(per_call),
            "calls": len(per_call), "calls_per_step": calls, "step_ms": step_ms,
            "sample": sample, "threads": threads}


def cpu_measure(name, budget_s):
    """(value, sample, threads) of `name`'s CPU restatement over ~budget_s."""
    r = cpu_bench(name, budget_s)
    return r["value"], f"{r['sample']}; {r['calls']} calls, median call time", r["threads"]


# ---------------------------------------------------------------------------- main
class stdout_to_stderr:
    """Points file descriptor 1 at stderr for the duration of the block."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    """The reference arm: the CPU restatement of the reference kernels'
    algorithm (oracle/, C OpenMP + numpy/OpenBLAS on every host thread) on the
    same workload as this repo's arm. For the softmax headline each call is
    the full 4096 x 16384 config, inputs built once before the timing."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O

    O.build()
    # torchrun sets OMP_NUM_THREADS=1 for its ranks; the CPU reference uses every
    # host thread this process may run on (OpenMP in the C port, the BLAS pool for numpy).
    ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    O.set_threads(ncpu)
    blas_threads = None
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        blas_limit = threadpool_limits(limits=ncpu, user_api="blas")
        blas_threads = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
    except Exception:  # threadpoolctl absent: BLAS keeps its own default
        blas_limit = None
    name = args.workload
    desc, unit, _, _ = WORKLOADS[name]
    budget = max(1.0, min(60.0, args.ref_budget))
    r = cpu_bench(name, budget, steps=args.steps, warmup=args.warmup)
    if blas_limit is not None:
        blas_limit.restore_original_limits()
    value = r["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.mean(r["step_ms"]), 3),
        "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f32" if unit == "GB/s" else "f16",
        "data": "synthetic",
        "config": {"workload": desc, "config_index": 1 if name == "softmax" else None},
        "parallelism": "host threads (rank 0 only)",
        "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": r["threads"],
                         "kind": "port",
                         "sample": (f"{r['sample']}; {r['calls_per_step']} calls per step, "
                                    f"value from the median call time")},
        "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "rate_min_time": round(r["best"], 3), "rate_mean_time": round(r["mean"], 3),
        "threads": {"openmp": O.threads(), "blas": blas_threads},
        "note": ("reference = CPU restatement of the reference kernels' algorithm (oracle/, "
                 "C OpenMP + numpy/OpenBLAS); Julia/cuTile/triton 3.7.1 are not installable here"),
    }
    print(json.dumps(line), flush=True)
    return 0


# bench/examples.jl names and implementation labels of the suite workloads.
RESULT_NAMES = {"vadd": ("vadd", "b200"), "rowsum": ("rowsum", "b200"),
                "softmax": ("softmax", "b200"), "layernorm": ("layernorm", "b200 Fwd"),
                "layernorm_bwd": ("layernorm", "b200 Bwd"),
                "layernorm_bwd_noalloc": ("layernorm", "b200 Bwd noalloc"),
                "transpose": ("transpose", "b200"),
                "gemm": ("matmul", "b200"), "bgemm": ("batchmatmul", "b200"),
                "fmha": ("fmha", "b200"), "fmha_causal": ("fmha", "b200 causal"),
                "moe": ("moe", "b200")}


def result_row(name, ms_min, ms_mean, work=None):
    """One `RESULT` row of bench/examples.jl:51: name, impl, min ms, mean ms and
    the rate from the minimum time (integer GB/s or TFLOPS to one decimal)."""
    ex, impl = RESULT_NAMES[name]
    _, unit, _, w = WORKLOADS[name]
    w = w if work is None else work
    if unit == "GB/s":
        metr = f"{round(w / (ms_min / 1e3) / 1e9)} GB/s"
    else:
        metr = f"{round(w / (ms_min / 1e3) / 1e12, 1)} TFLOPS"
    return f"RESULT\t{ex}\t{impl}\t{round(ms_min, 4)}\t{round(ms_mean, 4)}\t{metr}"


def _gpu_uuid(dev):
    import torch

    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


def run_ours(args):
    import torch

    world, rank, local = dist_env()
    dist_on = world > 1
    if dist_on:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL announces its version on stdout at communicator set-up; keep
        # stdout for the single JSON line.
        with stdout_to_stderr():
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import cutile_b200
    from cutile_b200 import ops

    ops.init(local)
    peaks, peak_src = load_peaks()
    traffic = load_traffic()
    strong = args.scaling == "strong"
    # Every rank samples its own GPU's clocks (per-rank medians name a rank
    # that runs slower); rank 0's samples are the line's `clocks`.
    sampler = ClockSampler(_gpu_uuid(dev) or local)
    sampler.start()
    flush = None  # allocated on first need: 256 MiB, twice the L2

    def measure(name, steps, warmup, want_e2e, want_cpu, cpu_budget, part_mode):
        nonlocal flush
        part = (rank, world) if part_mode else None
        case = Case(name, dev, rank, part=part)
        fl = None
        if case.bytes_in() + case.bytes_out() < 2 * L2_BYTES:
            if flush is None:
                flush = torch.zeros(2 * L2_BYTES // 4 // 4096, 4096, dtype=torch.float32,
                                    device=dev)
            fl = flush
        torch.cuda.synchronize()
        total_ms, mean_ms = time_device(case, steps, warmup, dist_on, fl)
        ops.check_device()
        _, unit, bound, work = WORKLOADS[name]
        scale = 1e9 if unit == "GB/s" else 1e12
        # strong: the ranks share ONE job of `work`; weak: each rank does a job.
        job = work if part_mode else world * work
        value = job * steps / (total_ms * 1e-3) / scale
        rank_work = work * case.units / case.total_units if part_mode else work
        res = {"value": round(value, 3), "unit": unit, "ms_per_step": round(total_ms / steps, 5),
               "roofline": roofline(name, mean_ms, peaks, peak_src, traffic, rank_work),
               "gpu_launches": steps * LAUNCHES_PER_STEP.get(name, 1),
               "launch_ms": case.launch_stats, "rank_launch_ms": round(case.rank_launch_ms, 5),
               "dtype": "f16" if bound == "tensor" else "f32",
               "l2": (f"{case.bytes_in() / 1e6:.0f} MB read + {case.bytes_out() / 1e6:.0f} MB "
                      f"written per step per rank; "
                      + ("L2 flushed (256 MiB read) before every timed launch" if fl is not None
                         else "larger than L2 (126 MB), no flush"))}
        if want_e2e:
            k = max(2, min(steps, 10))
            ms, bi, bo = time_e2e(case, k, dev, dist_on)
            res["e2e"] = {"value": round(job / (ms * 1e-3) / scale, 3), "unit": unit,
                          "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo}
        case.free()
        del case
        torch.cuda.empty_cache()
        if want_cpu and rank == 0 and world == 1:
            r = cpu_bench(name, cpu_budget, steps=1, warmup=1)
            res["cpu_baseline"] = {"value": round(r["value"], 3), "unit": unit,
                                   "cores": r["threads"], "kind": "port",
                                   "sample": (f"{r['sample']}; {r['calls']} calls, value from "
                                              f"the median call time")}
        return res

    head = args.workload
    desc = WORKLOADS[head][0]
    h = measure(head, args.steps, args.warmup, True, True, args.cpu_budget, strong)
    weak = None
    if dist_on and strong:
        # The second scaling number: every rank a full config of its own.
        w = measure(head, args.steps, args.warmup, False, False, 0, False)
        weak = {"value": w["value"], "ms_per_step": w["ms_per_step"],
                "frac_per_gpu": w["roofline"]["frac"], "scaling": "weak"}
    suite = {}
    if args.suite:
        for name in SUITE_ORDER:
            if name == head:
                continue
            steps = args.suite_steps if not name.startswith("fmha") else max(3, args.suite_steps // 4)
            full = name not in NO_E2E_CPU
            suite[name] = measure(name, steps, max(3, args.warmup), full,
                                  full, args.cpu_budget / 3, strong)
            suite[name]["config"] = WORKLOADS[name][0]
    gather = None
    if args.gather and dist_on:
        # Optional final gather of every rank's headline output (NCCL over
        # NVLink/NVSwitch), after and apart from the timed kernels.
        import torch.distributed as dist
        from cutile_b200.shard import gather_shards

        gcase = Case(head, dev, rank)
        gcase.run()
        out = gcase.outputs[0]
        gather_shards(out)  # warm-up (communicator buffers)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        full = gather_shards(out)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nbytes = out.numel() * out.element_size()
        gather = {"what": f"all-gather of each rank's {head} output", "bytes_per_rank": nbytes,
                  "bytes_total": full.numel() * full.element_size(), "ms": round(t.item(), 4),
                  "GB/s_received_per_rank": round(nbytes * (world - 1) / (t.item() * 1e-3) / 1e9, 1)}
        del full, gcase
        torch.cuda.empty_cache()
    lp = launch_path(dev) if (args.suite and rank == 0) else None
    sampler.stop()
    clocks = sampler.summary()
    per_rank = None
    if dist_on:
        import torch.distributed as dist

        mine = {"rank": rank, "gpu": _gpu_uuid(dev), "sm_mhz": clocks["sm_mhz"],
                "reasons": clocks["reasons"], "launch_ms": {head: h["rank_launch_ms"],
                **{k: v["rank_launch_ms"] for k, v in suite.items()}}}
        allr = [None] * world
        dist.all_gather_object(allr, mine)
        per_rank = {"sm_mhz": [r["sm_mhz"] for r in allr],
                    "reasons": sorted({x for r in allr for x in r["reasons"]}),
                    "launch_ms": {k: [r["launch_ms"][k] for r in allr]
                                  for k in allr[0]["launch_ms"]}}
    if rank == 0:
        roof = {k: v for k, v in h["roofline"].items() if k != "peak_source"}
        rows = {head: h, **suite}
        detail = {"headline": h, "suite": suite, "weak": weak, "per_rank": per_rank,
                  "launch_path": lp, "gather": gather, "clocks": clocks,
                  "library": cutile_b200.library_path(), "peaks": peak_src}
        if args.detail:
            with open(args.detail, "w") as f:
                json.dump(detail, f, indent=1)
        print("DETAIL " + json.dumps(detail), file=sys.stderr, flush=True)
        if args.result_rows:
            for name in SUITE_ORDER:
                if name in rows:
                    lm = rows[name]["launch_ms"]
                    print(result_row(name, lm["ms_min"], lm["ms_mean"],
                                     rows[name]["roofline"]["algorithmic_per_launch"]), flush=True)
        line = {
            "metric": METRIC, "value": h["value"], "unit": h["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": h["ms_per_step"],
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": h["dtype"],
            "data": "synthetic (seeded SplitMix64, BASELINE shapes and distributions)",
            "config": {"workload": desc, "config_index": 1 if head == "softmax" else None},
            "parallelism": (f"dp{world}, " + ("one job split by rows over the ranks" if strong
                                              else "each rank a full config")),
            "l2": h["l2"],
            "roofline": roof, "cpu_baseline": h.get("cpu_baseline"),
            "e2e": h.get("e2e"), "gpu_launches": h["gpu_launches"],
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            **({"weak": weak} if weak else {}),
            **({"per_rank": per_rank} if per_rank else {}),
            "suite_fields": ["value", "roofline.frac", "e2e.value", "cpu_baseline.value",
                             "gpu_launches"],
            "suite": {k: [v["value"], v["roofline"]["frac"], (v.get("e2e") or {}).get("value"),
                          (v.get("cpu_baseline") or {}).get("value"), v["gpu_launches"]]
                      for k, v in suite.items()},
        }
        print(json.dumps(line), flush=True)
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_profile(args):
    """Runs W warm-up launches and K launches of one workload, nothing else:
    the command under ncu captures (`--profile NAME`, small inputs for vadd
    and fmha so that a multi-pass capture stays a few GB and seconds)."""
    import torch

    from cutile_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops.init(0)
    case = Case(args.profile, dev, 0, small=not args.full_size)
    for _ in range(args.warmup + args.steps):
        case.run()
    torch.cuda.synchronize()
    ops.check_device()
    print(f"profile case {args.profile}: {args.warmup} + {args.steps} launches ok")
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="softmax", choices=list(WORKLOADS))
    ap.add_argument("--suite", dest="suite", action="store_true", default=True)
    ap.add_argument("--no-suite", dest="suite", action="store_false")
    ap.add_argument("--suite-steps", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=10.0,
                    help="seconds of CPU work for the headline cpu_baseline")
    ap.add_argument("--ref-budget", type=float, default=12.0,
                    help="seconds of CPU work for the reference arm (all steps together)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="N>1: split one BASELINE job over the ranks (strong, the default; the "
                         "headline's weak number is added) or give every rank a full job (weak)")
    ap.add_argument("--result-rows", action="store_true",
                    help="also print bench/examples.jl's RESULT rows (before the JSON line)")
    ap.add_argument("--detail", default=None, help="write every measured figure to this JSON file")
    ap.add_argument("--gather", action="store_true",
                    help="under torchrun: also time an all-gather of the headline output (NCCL)")
    ap.add_argument("--full-size", action="store_true",
                    help="with --profile: the bench's own sizes instead of the small case")
    ap.add_argument("--profile", default=None, choices=list(WORKLOADS),
                    help="launch-only mode for ncu captures")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # the timing rules require >= 3 warm-up steps
    if args.profile:
        return run_profile(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
