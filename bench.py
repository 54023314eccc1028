"""Benchmark of the ThunderKittens-SM7x hot path on B200 (one process per GPU).

Headline step (per GPU, weak scaling): one FP16 x FP16 -> FP32 GEMM of
8192 x 8192 x 8192 (this rank's 8192-row block of an (8192 * N)-row A, with B
replicated), one attention forward over [8, 32, 4096, 128] unmasked and one causal
(this rank's batch x head shard). value = all FLOPs of all ranks / max-over-ranks
device time, in TFLOP/s.

The same JSON line also carries, as `configs`, one measurement per other benchmark
configuration of the path (N = 1): GEMM 256^3, the 1,048,576-tile row ops (each op
and all four fused), the fused row-statistics and row-softmax GEMMs at 8192^3, the
padded 16384 x 4096 x 14336 GEMM, the decode-shaped 16 x 4096 x 4096 GEMM and the
one-tile attention; and at N > 1, as `multi_gpu`, the fixed-size (strong scaling)
GEMM, attention and row ops split across the ranks, the gathered outputs (GEMM with
the all-gather fused into its epilogue, or GEMM / attention followed by an NCCL
all-gather), and the hosts' copy bandwidth with every rank copying at once.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload headline|gemm|attention|rowops] [--gather [fused|nccl]]
                    [--no-configs] [--no-cpu-baseline]
    python bench.py --sustained SECONDS   # power-capped rates, ours beside cuBLAS / cuDNN

Timing: K steps between two CUDA events on the launching stream, a barrier and
torch.cuda.synchronize() on both sides, the max over ranks. Headline inputs are
larger than L2 (126 MB); configurations whose inputs fit in L2 (256^3, the decode
GEMM, the one-tile attention) are timed one call at a time with a 256 MiB buffer
written between calls. Fractions of the tensor peak use the measured burst bf16
rate when the timed region lasts under a second, else the sustained one. e2e repeats
the step through the same C ABI with host buffers: pinned host -> device copies of
the step's inputs and device -> host copies of its outputs inside the timed region.

--impl reference times the reference's CPU implementation of the path on bounded
row samples with all host threads, on rank 0 only: its FP64 host GEMM oracle
compiled from its sources (oracle/_ref, "reference") and the generalised FP64
attention oracle restated from its one-tile host oracle ("port"); the same samples
as the `cpu_baseline` leg of our arm.
"""

from __future__ import annotations

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
sys.path[:0] = [ROOT, os.path.join(ROOT, "thunderkittens-sm7x_b200")]

GEMM_M = GEMM_N = GEMM_K = 8192
ATT_B, ATT_H, ATT_S, ATT_D = 8, 32, 4096, 128
ROW_TILES = 1 << 20

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def gemm_flops(m=GEMM_M, n=GEMM_N, k=GEMM_K):
    return 2.0 * m * n * k


def attn_flops(causal, b=ATT_B, h=ATT_H, s=ATT_S, d=ATT_D):
    if causal:
        return 4.0 * b * h * d * s * (s + 1) / 2
    return 4.0 * b * h * s * s * d


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def tensor_peak(peaks, timed_seconds):
    """(peak TFLOP/s, key): the burst cuBLAS rate for a timed region under a second
    (the clock has not yet settled under the power cap), the sustained one above."""
    key = "bf16_tflops" if timed_seconds < 1.0 else "bf16_tflops_sustained"
    return peaks.get(key, FALLBACK_PEAKS[key]), key


def load_traffic():
    """Per-launch DRAM bytes from a committed ncu summary (profiles/ncu_traffic.json)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._reader = threading.Thread(target=self._read, daemon=True)
            self._reader.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._reader.join(timeout=5)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def init_dist():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------------

class Workload:
    """Device-resident inputs and the list of (name, launch, flops_or_bytes) calls of one step."""

    def __init__(self, kind: str, rank: int, world: int, row_tiles: int = ROW_TILES, fused_gather: bool = False):
        import torch
        import tk_b200
        self.kind = kind
        self.tk = tk_b200
        gen = torch.Generator(device="cuda")
        self.calls = []
        self.h2d = []   # (device tensor) inputs copied in per e2e step
        self.d2h = []   # (device tensor) outputs copied out per e2e step
        self.gathered = []  # outputs already gathered by their kernel (fused all-gather)
        self.gbuf = None
        if kind in ("headline", "gemm"):
            gen.manual_seed(2 + 1000 * rank)
            self.a = (torch.rand(GEMM_M, GEMM_K, device="cuda", generator=gen) * 2 - 1).half()
            gen.manual_seed(2)
            self.b = (torch.rand(GEMM_K, GEMM_N, device="cuda", generator=gen) * 2 - 1).half()
            if fused_gather and world > 1:
                # Every rank's 8192-row block lands in every rank's gathered C from the
                # GEMM epilogue (NVLink stores), no separate collective.
                from tk_b200 import dist as tkd
                self.gbuf = tkd.GatheredBuffer(world * GEMM_M, GEMM_N)
                self.c = self.gbuf.tensor()[rank * GEMM_M:(rank + 1) * GEMM_M]
                self.calls.append(("gemm_8192", lambda: self.tk.gemm_gather_raw(
                    GEMM_M, GEMM_N, GEMM_K, self.a, GEMM_K, self.b, GEMM_N, self.gbuf.ptrs, rank, GEMM_N),
                    gemm_flops(), 1))
                self.gathered.append(self.c)
            else:
                self.c = torch.empty(GEMM_M, GEMM_N, device="cuda")
                self.calls.append(("gemm_8192", lambda: self.tk.gemm_raw(
                    GEMM_M, GEMM_N, GEMM_K, self.a, GEMM_K, self.b, GEMM_N, self.c, GEMM_N), gemm_flops(), 1))
            self.h2d += [self.a, self.b]
            self.d2h += [self.c]
        if kind in ("headline", "attention"):
            gen.manual_seed(4 + 1000 * rank)
            shape = (ATT_B, ATT_H, ATT_S, ATT_D)
            self.q = torch.randn(shape, device="cuda", generator=gen).half()
            self.k = torch.randn(shape, device="cuda", generator=gen).half()
            self.v = torch.randn(shape, device="cuda", generator=gen).half()
            self.o = torch.empty(shape, device="cuda")
            self.oc = torch.empty(shape, device="cuda")
            scale = 1.0 / math.sqrt(ATT_D)
            self.calls.append(("attention_fwd", lambda: self.tk.attention_raw(
                self.q, self.k, self.v, self.o, ATT_B, ATT_H, ATT_S, ATT_D, scale, False), attn_flops(False), 1))
            self.calls.append(("attention_fwd_causal", lambda: self.tk.attention_raw(
                self.q, self.k, self.v, self.oc, ATT_B, ATT_H, ATT_S, ATT_D, scale, True), attn_flops(True), 1))
            self.h2d += [self.q, self.k, self.v]
            self.d2h += [self.o, self.oc]
        if kind == "rowops":
            gen.manual_seed(1 + 1000 * rank)
            self.tiles = torch.randn(row_tiles * 256, device="cuda", generator=gen) * 2
            self.rs = torch.empty(row_tiles * 16, device="cuda")
            self.rm = torch.empty(row_tiles * 16, device="cuda")
            self.sm = torch.empty(row_tiles * 256, device="cuda")
            self.cs = torch.empty(row_tiles * 256, device="cuda")
            nbytes = row_tiles * 1024 * 3 + row_tiles * 128
            self.calls.append(("tile_row_ops_all4", lambda: self.tk.row_ops_raw(
                self.tiles, row_tiles, self.rs, self.rm, self.sm, self.cs), float(nbytes), 1))
            self.h2d += [self.tiles]
            self.d2h += [self.rs, self.rm, self.sm, self.cs]

    @property
    def call_meta(self):
        return self._meta

    def freeze(self):
        """Records (name, work) of the step's calls and its launches per step."""
        self._meta = [(c[0], c[2]) for c in self.calls]
        self.launches_per_step = sum(c[3] for c in self.calls)

    def step(self, events=None):
        for i, (name, fn, _, _) in enumerate(self.calls):
            if events is not None:
                events[i][0].record()
            code = fn()
            if code != 0:
                raise RuntimeError(f"{name} failed with cudaError {code}")
            if events is not None:
                events[i][1].record()


def run_ours(args, rank, world, local):
    import torch
    import tk_b200
    tk_b200.lib().tk_attention_set_cta_group(2 if args.attention_kernel == "pair" else 1)
    fused = args.gather == "fused"
    wl = Workload(args.workload, rank, world, args.row_tiles, fused_gather=fused)
    wl.freeze()
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()

    ncalls = len(wl.calls)
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(ncalls)]
          for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    for s in range(args.steps):
        wl.step(ev[s])
        if args.gather and world > 1:
            gather_outputs(wl, world)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)

    per_kernel_ms = [sum(ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps)) / args.steps
                     for i in range(ncalls)]
    per_kernel_ms = [max_over_ranks(x, world) for x in per_kernel_ms]
    work_per_step = sum(c[2] for c in wl.calls) * world
    ms_per_step = elapsed_ms / args.steps

    # e2e: host buffers through the same C ABI, every step's inputs copied in from
    # pinned host memory and its outputs copied back inside the timed region. Two
    # device buffer sets and separate copy streams let step i's kernels overlap the
    # host->device copy of step i+1 and the device->host copy of step i-1 (the PCIe
    # directions are independent), as a pipelined host application would run.
    wl2 = Workload(args.workload, rank, world, args.row_tiles, fused_gather=fused)
    wl2.freeze()
    sets = [wl, wl2]
    # One pinned host copy of the inputs and one of the outputs serve both device
    # sets: copies in one direction are serialised on their stream.
    host_in_set = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in wl.h2d]
    host_out_set = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in wl.d2h]
    for h, d in zip(host_in_set, wl.h2d):
        h.copy_(d)
    host_in = [host_in_set, host_in_set]
    host_out = [host_out_set, host_out_set]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    # The same K steps as the device-resident timing (at least 4): the pipeline's
    # fill (the first inputs in) and drain (the last outputs out) count once per run,
    # as they do for a host application streaming K batches.
    e2e_steps = max(4, args.steps)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    comp_done = [None, None]
    out_done = [None, None]
    for i in range(e2e_steps):
        b = i % 2
        w = sets[b]
        with torch.cuda.stream(s_in):
            if comp_done[b] is not None:
                s_in.wait_event(comp_done[b])       # step i-2 finished reading these inputs
            for h, d in zip(host_in[b], w.h2d):
                d.copy_(h, non_blocking=True)
            in_ready = torch.cuda.Event()
            in_ready.record(s_in)
        comp.wait_event(in_ready)
        if out_done[b] is not None:
            comp.wait_event(out_done[b])            # step i-2's outputs are on the host
        w.step()
        done = torch.cuda.Event()
        done.record(comp)
        comp_done[b] = done
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for h, d in zip(host_out[b], w.d2h):
                h.copy_(d, non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(s_out)
            out_done[b] = copied
    for ev in out_done:
        if ev is not None:
            comp.wait_event(ev)
    e1.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / e2e_steps
    h2d_bytes = sum(t.numel() * t.element_size() for t in wl.h2d)
    d2h_bytes = sum(t.numel() * t.element_size() for t in wl.d2h)
    if wl2.gbuf is not None:
        wl2.gbuf.close()  # collective
    del wl2, host_in, host_out, host_in_set, host_out_set

    status = wl.tk.device_status()
    if status != 0:
        raise RuntimeError(f"kernel status word {status:#x}: a bounded wait gave up")
    return wl, ms_per_step, per_kernel_ms, work_per_step, clocks, e2e_ms, h2d_bytes, d2h_bytes


def gather_outputs(wl, world):
    """NCCL all-gather of this step's outputs not already gathered by their kernel
    (only with --gather)."""
    import torch
    import torch.distributed as dist
    for t in wl.d2h:
        if any(t is g for g in wl.gathered):
            continue
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t)


def cpu_sample_gemm(threads: int, rows_per_thread: int = 2, cols: int = 1024):
    """FP64 GEMM oracle on a sample of the 8192^3 workload (rows x the first `cols`
    columns, all of K). Prefers the reference's own host code (oracle/_ref), else
    the restated oracle."""
    import ctypes as C

    import numpy as np

    import oracle
    ldb = k = GEMM_K
    n = cols
    rows = threads * rows_per_thread
    a = np.zeros((rows, k), np.uint16)
    b = np.zeros((k, ldb), np.uint16)
    oracle.lib().tko_gen_gemm_uniform(2, -1.0, 1.0, rows, ldb, k, a.reshape(-1), k, b.reshape(-1), ldb)
    ref = oracle.ref_lib()
    kind = "reference" if ref is not None else "port"

    def work(i):
        blk = np.ascontiguousarray(a[i * rows_per_thread:(i + 1) * rows_per_thread])
        m = blk.shape[0]
        if ref is not None:
            val = np.empty((m, n))
            sa = np.empty((m, n))
            bd = np.empty((m, n))
            p = lambda x: x.ctypes.data_as(C.c_void_p)  # noqa: E731
            ref.tkref_diff_reference(m, n, k, k, ldb, n, 0, 1, p(blk), p(b), p(val), p(sa), p(bd))
        else:
            oracle.gemm_ref(m, n, k, blk, k, b, ldb)

    t0 = time.perf_counter()
    ts = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    dt = time.perf_counter() - t0
    return (gemm_flops(rows, n, k), dt, kind,
            f"{rows} rows x {n} columns x K 8192 (FP64 host GEMM with |a.b| sums)")


def cpu_sample_attention(threads: int, rows_per_thread: int, causal: bool):
    import numpy as np

    import oracle
    count = ATT_S * ATT_D
    q, k, v = oracle.gen_qkv_normal(4, 1.0, count)  # one (batch, head) slice

    def work(i):
        # Query rows from the end of the sequence (the full key range); threads past
        # the slice wrap around.
        lo = (ATT_S - (i + 1) * rows_per_thread) % ATT_S
        lo = min(lo, ATT_S - rows_per_thread)
        oracle.attention_ref(q, k, v, ATT_S, ATT_D, 1 / math.sqrt(ATT_D), causal, lo, lo + rows_per_thread)

    t0 = time.perf_counter()
    ts = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    dt = time.perf_counter() - t0
    rows = threads * rows_per_thread
    flops = 4.0 * rows * ATT_S * ATT_D
    return flops, dt, f"{rows} query rows x 4096 keys x 128 (FP64 attention, P rounded to FP16)"


# Rows per host thread of the CPU samples, shared by the cpu_baseline leg of our arm
# and every step of the reference arm (the same sample in both).
CPU_GEMM_ROWS, CPU_ATTN_ROWS = 4, 128


def cpu_baseline(threads: int, workload: str, gemm_rows: int = CPU_GEMM_ROWS, attn_rows: int = CPU_ATTN_ROWS):
    """Returns (TFLOP/s over the sampled work, kind, description, seconds, legs) for the
    step's FLOP mix: legs maps each sampled kernel to "reference" (the reference's own
    host code, oracle/_ref) or "port" (the restated oracle); kind is "reference" only
    when every leg is."""
    parts = []
    legs = {}
    if workload in ("headline", "gemm"):
        f, dt, kind_g, desc = cpu_sample_gemm(threads, rows_per_thread=gemm_rows)
        parts.append((f, dt, desc))
        legs["gemm"] = kind_g
    if workload in ("headline", "attention"):
        f, dt, desc = cpu_sample_attention(threads, min(attn_rows, ATT_S), False)
        parts.append((f, dt, desc))
        legs["attention"] = "port"  # the reference's host attention oracle is fixed at 16 x 16
    if not parts:
        return None
    kind = "reference" if all(v == "reference" for v in legs.values()) else "port"
    # Time the sampled work of each kernel and scale to the step's FLOP mix.
    step_mix = {"headline": [gemm_flops(), attn_flops(False) + attn_flops(True)],
                "gemm": [gemm_flops()], "attention": [attn_flops(False) + attn_flops(True)]}[workload]
    step_seconds = sum(mix / (f / dt) for mix, (f, dt, _) in zip(step_mix, parts))
    tflops = sum(step_mix) / step_seconds / 1e12
    sample = "; ".join(d for _, _, d in parts)
    return tflops, kind, sample, sum(dt for _, dt, _ in parts), legs


# ---------------------------------------------------------------------------------
# Per-configuration measurements (single GPU) and multi-GPU components
# ---------------------------------------------------------------------------------

class L2Flush:
    """A 256 MiB device buffer (twice the 126 MB L2) written, then read, between timed
    calls whose inputs would otherwise stay in L2. The read leaves clean lines, so the
    timed call does not pay for writing back the flush's own dirty lines."""

    def __init__(self):
        import torch
        self.buf = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
        self.sink = torch.empty((), dtype=torch.float32, device="cuda")

    def __call__(self):
        import torch
        self.buf.zero_()
        torch.sum(self.buf, dim=0, out=self.sink)


def graph_per_call_us(fn, calls=256):
    """Device time per call (us) of `calls` back-to-back calls captured in one CUDA graph
    and replayed: launch-to-launch cost on the GPU without the host's per-call cost
    (what the reference's benchmarks count for its latency-bound entry points)."""
    import torch
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(calls):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    for _ in range(5):
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e3 / calls
        best = t if best is None else min(best, t)
    del g
    return best


def time_calls(fn, iters, flush=None, warmup=3):
    """Median and minimum device time (ms) of `fn()` over `iters` calls, each between
    CUDA events on the current stream; `flush` (if given) runs before every call,
    outside the events. fn returns a cudaError code (0 = success)."""
    import torch
    for _ in range(warmup):
        if flush:
            flush()
        code = fn()
        if code != 0:
            raise RuntimeError(f"call failed with cudaError {code}")
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for e0, e1 in evs:
        if flush:
            flush()
        e0.record()
        fn()
        e1.record()
    torch.cuda.synchronize()
    ts = sorted(e0.elapsed_time(e1) for e0, e1 in evs)
    return ts[len(ts) // 2], ts[0]


def run_configs(peaks, traffic, iters=20):
    """One entry per benchmark configuration other than the headline step (per GPU).
    Work per call and the bound come from the configuration's algorithmic FLOPs or
    bytes; frac is against the measured burst bf16 rate (tensor-bound calls, each
    timed alone) or the measured HBM copy bandwidth (HBM-bound calls)."""
    import torch
    import tk_b200
    gen = torch.Generator(device="cuda")
    flush = L2Flush()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    burst = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    out = {}

    def tensor_entry(ms, flop, extra=None):
        rate = flop / (ms / 1e3) / 1e12
        e = {"ms": round(ms, 4), "TFLOP/s": round(rate, 1), "frac": round(rate / burst, 4), "bound": "tensor",
             "peak": f"measured bf16_tflops {burst}"}
        e.update(extra or {})
        return e

    def hbm_entry(ms, nbytes, extra=None):
        rate = nbytes / (ms / 1e3) / 1e9
        e = {"ms": round(ms, 4), "GB/s": round(rate, 1), "frac": round(rate / hbm, 4), "bound": "hbm",
             "bytes": int(nbytes), "peak": f"measured hbm_gbs {hbm}"}
        e.update(extra or {})
        return e

    # cfg1: GEMM 256^3 (U[-1, 1], seed 0), lda = ldb = ldc = 256: a latency-bound call.
    gen.manual_seed(0)
    a = (torch.rand(256, 256, device="cuda", generator=gen) * 2 - 1).half()
    b = (torch.rand(256, 256, device="cuda", generator=gen) * 2 - 1).half()
    c = torch.empty(256, 256, device="cuda")
    med, best = time_calls(lambda: tk_b200.gemm_raw(256, 256, 256, a, 256, b, 256, c, 256), iters, flush)
    b2b = graph_per_call_us(lambda: tk_b200.gemm_raw(256, 256, 256, a, 256, b, 256, c, 256,
                                                     torch.cuda.current_stream()))
    out["gemm_256"] = tensor_entry(med, gemm_flops(256, 256, 256),
                                   {"us_per_call": round(med * 1e3, 2), "us_per_call_back_to_back": round(b2b, 2),
                                    "timing": "us_per_call: one call, L2 and TLB cold (256 MiB written and read "
                                              "between calls); back to back: 256 calls in one CUDA graph"})
    del a, b, c

    # cfg2: 1,048,576 tiles of 16 x 16 FP32, N(0, 4) (seed 1): each op alone and all four fused.
    tiles = ROW_TILES
    gen.manual_seed(1)
    x = torch.randn(tiles * 256, device="cuda", generator=gen) * 2
    rs = torch.empty(tiles * 16, device="cuda")
    rm = torch.empty(tiles * 16, device="cuda")
    sm = torch.empty(tiles * 256, device="cuda")
    cs = torch.empty(tiles * 256, device="cuda")
    rin = tiles * 1024
    for name, kw, nbytes in [
            ("row_sum", {"row_sum": rs}, rin + tiles * 64),
            ("row_max", {"row_max": rm}, rin + tiles * 64),
            ("row_softmax", {"softmax": sm}, rin + tiles * 1024),
            ("row_softmax_causal", {"softmax_causal": cs}, rin + tiles * 1024),
            ("row_ops_all4", {"row_sum": rs, "row_max": rm, "softmax": sm, "softmax_causal": cs},
             rin + 2 * tiles * 64 + 2 * tiles * 1024)]:
        med, best = time_calls(lambda kw=kw: tk_b200.row_ops_raw(x, tiles, **kw), iters)
        extra = {"tiles": tiles}
        tr = traffic.get("tile_row_ops_all4" if name == "row_ops_all4" else name, {})
        if "dram_bytes_per_tile" in tr:
            extra["traffic"] = round(tr["dram_bytes_per_tile"] * tiles)
        out[f"rowops_{name}"] = hbm_entry(med, nbytes, extra)
    del x, rs, rm, sm, cs

    # cfg3 fused variants: GEMM 8192^3 with the row-statistics epilogue, and with the
    # full-row softmax (U[-1, 1], seed 2).
    gen.manual_seed(2)
    a = (torch.rand(GEMM_M, GEMM_K, device="cuda", generator=gen) * 2 - 1).half()
    b = (torch.rand(GEMM_K, GEMM_N, device="cuda", generator=gen) * 2 - 1).half()
    c = torch.empty(GEMM_M, GEMM_N, device="cuda")
    mx = torch.empty(GEMM_M, device="cuda")
    sm_ = torch.empty(GEMM_M, device="cuda")
    med, _ = time_calls(lambda: tk_b200.gemm_raw(GEMM_M, GEMM_N, GEMM_K, a, GEMM_K, b, GEMM_N, c, GEMM_N), iters)
    out["gemm_8192"] = tensor_entry(med, gemm_flops())
    med, _ = time_calls(lambda: tk_b200.gemm_rowstats_raw(GEMM_M, GEMM_N, GEMM_K, a, GEMM_K, b, GEMM_N, c, GEMM_N,
                                                          mx, sm_), iters)
    out["gemm_8192_rowstats"] = tensor_entry(med, gemm_flops(), {"outputs": "C + row_max + row_sum"})
    med, _ = time_calls(lambda: tk_b200.gemm_rowsoftmax_raw(GEMM_M, GEMM_N, GEMM_K, a, GEMM_K, b, GEMM_N, c, GEMM_N,
                                                            c, GEMM_N), iters)
    out["gemm_8192_rowsoftmax"] = tensor_entry(med, gemm_flops(), {"outputs": "P (softmax of C, in place)"})
    del a, b, c, mx, sm_

    # cfg4a: M = 16384, N = 4096, K = 14336, lda = K + 64, ldb = ldc = N + 32, N(0, 0.02^2) (seed 3).
    m4, n4, k4 = 16384, 4096, 14336
    lda, ldb, ldc = k4 + 64, n4 + 32, n4 + 32
    gen.manual_seed(3)
    a = (torch.randn(m4, lda, device="cuda", generator=gen) * 0.02).half()
    b = (torch.randn(k4, ldb, device="cuda", generator=gen) * 0.02).half()
    c = torch.empty(m4, ldc, device="cuda")
    med, _ = time_calls(lambda: tk_b200.gemm_raw(m4, n4, k4, a, lda, b, ldb, c, ldc), iters)
    out["gemm_16384x4096x14336_padded"] = tensor_entry(med, gemm_flops(m4, n4, k4),
                                                      {"lda": lda, "ldb": ldb, "ldc": ldc})
    del a, b, c

    # cfg4b: decode-shaped M = 16, N = K = 4096 (seed 3): HBM-bound (B is 32 MiB).
    gen.manual_seed(3)
    a = (torch.randn(16, 4096, device="cuda", generator=gen) * 0.02).half()
    b = (torch.randn(4096, 4096, device="cuda", generator=gen) * 0.02).half()
    c = torch.empty(16, 4096, device="cuda")
    med, _ = time_calls(lambda: tk_b200.gemm_raw(16, 4096, 4096, a, 4096, b, 4096, c, 4096), iters, flush)
    nbytes = 16 * 4096 * 2 + 4096 * 4096 * 2 + 16 * 4096 * 4
    b2b = graph_per_call_us(lambda: tk_b200.gemm_raw(16, 4096, 4096, a, 4096, b, 4096, c, 4096,
                                                     torch.cuda.current_stream()))
    out["gemm_16x4096x4096_decode"] = hbm_entry(med, nbytes, {"TFLOP/s": round(gemm_flops(16, 4096, 4096) / med / 1e9, 2),
                                                              "timing": "L2 flushed between calls",
                                                              "us_per_call": round(med * 1e3, 2),
                                                              "us_per_call_back_to_back_l2_resident": round(b2b, 2),
                                                              "kernel": "operand-swapped small-M kernel"})
    # The same call on 128-row tiles (the path the operand-swapped kernel replaces), for comparison.
    prev = tk_b200.lib().tk_gemm_set_small_m(0)
    try:
        med0, _ = time_calls(lambda: tk_b200.gemm_raw(16, 4096, 4096, a, 4096, b, 4096, c, 4096), iters, flush)
    finally:
        tk_b200.lib().tk_gemm_set_small_m(prev)
    out["gemm_16x4096x4096_decode_row_tiles"] = hbm_entry(med0, nbytes, {"us_per_call": round(med0 * 1e3, 2),
                                                                         "timing": "L2 flushed between calls",
                                                                         "kernel": "128-row tiles, split-K"})
    del a, b, c

    # cfg5a: the one-tile attention (16 x 16, scale 1/4, N(0, 1), seed 4), unmasked and causal.
    gen.manual_seed(4)
    q = torch.randn(16, 16, device="cuda", generator=gen).half()
    k = torch.randn(16, 16, device="cuda", generator=gen).half()
    v = torch.randn(16, 16, device="cuda", generator=gen).half()
    o = torch.empty(16, 16, device="cuda")
    for causal in (False, True):
        med, _ = time_calls(lambda causal=causal: tk_b200.attention_16x16_raw(q, k, v, o, causal), iters, flush)
        b2b = graph_per_call_us(lambda causal=causal: tk_b200.attention_16x16_raw(q, k, v, o, causal,
                                                                                  torch.cuda.current_stream()))
        out["attention_16x16" + ("_causal" if causal else "")] = {
            "bound": "latency", "us_per_call": round(med * 1e3, 2), "us_per_call_back_to_back": round(b2b, 2),
            "timing": "us_per_call: one call, L2 and TLB cold (256 MiB written and read between calls); back to "
                      "back: 256 public calls in one CUDA graph (the reference's benchmark counts 2048 back-to-back "
                      "launches)"}
    del flush
    return out


def host_link(rank, world, h2d_tensors, d2h_tensors, reps=3):
    """Pinned host <-> device copy bandwidth with every rank copying at once: the step's
    inputs in and its outputs out, the two directions on separate streams. Returns the
    per-rank and aggregate GB/s (max over ranks of the time)."""
    import torch
    hin = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in h2d_tensors]
    hout = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in d2h_tensors]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    nbytes = sum(t.numel() * t.element_size() for t in h2d_tensors + d2h_tensors)
    best = None
    for _ in range(reps):
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        s_in.wait_event(e0)
        s_out.wait_event(e0)
        with torch.cuda.stream(s_in):
            for h, d in zip(hin, h2d_tensors):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            for h, d in zip(hout, d2h_tensors):
                h.copy_(d, non_blocking=True)
        torch.cuda.current_stream().wait_stream(s_in)
        torch.cuda.current_stream().wait_stream(s_out)
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), world)
        best = ms if best is None else min(best, ms)
    del hin, hout
    per_rank = nbytes / (best / 1e3) / 1e9
    return {"bytes_per_rank": nbytes, "ms": round(best, 3), "GB/s_per_rank": round(per_rank, 1),
            "GB/s_aggregate": round(per_rank * world, 1), "ranks_copying": world}


def run_multi_gpu(rank, world, peaks, iters=10):
    """Fixed-size problems split across the ranks (strong scaling) and gathered outputs.
    Every rank takes the same collective steps in the same order. Times are per call,
    between CUDA events after a barrier, max over ranks."""
    import torch
    import torch.distributed as dist
    import tk_b200
    from tk_b200 import dist as tkd
    gen = torch.Generator(device="cuda")
    burst = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    out = {}

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            barrier(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        return max_over_ranks(ts[len(ts) // 2], world)

    def check(code):
        if code != 0:
            raise RuntimeError(f"call failed with cudaError {code}")

    # GEMM 8192^3 split by M: rank r computes rows [r0, r1) of C; B replicated.
    r0, r1 = tkd.gemm_rows(GEMM_M, world, rank)
    rows = r1 - r0
    gen.manual_seed(2)
    a_full = (torch.rand(GEMM_M, GEMM_K, device="cuda", generator=gen) * 2 - 1).half()
    b = (torch.rand(GEMM_K, GEMM_N, device="cuda", generator=gen) * 2 - 1).half()
    a = a_full[r0:r1].contiguous()
    del a_full
    c = torch.empty(rows, GEMM_N, device="cuda")
    ms = timed(lambda: check(tk_b200.gemm_raw(rows, GEMM_N, GEMM_K, a, GEMM_K, b, GEMM_N, c, GEMM_N)))
    tf = gemm_flops() / (ms / 1e3) / 1e12
    out["gemm_8192_strong"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "frac_per_gpu": round(tf / world / burst, 4),
                               "rows_per_rank": rows}
    # ... with C gathered on every rank: fused into the GEMM epilogue (stores into every
    # rank's IPC-mapped buffer over NVLink), or the GEMM then an NCCL all-gather.
    gbuf = tkd.GatheredBuffer(GEMM_M, GEMM_N)
    ms = timed(lambda: check(tk_b200.gemm_gather_raw(rows, GEMM_N, GEMM_K, a, GEMM_K, b, GEMM_N, gbuf.ptrs, rank,
                                                     GEMM_N)))
    link = (world - 1) * rows * GEMM_N * 4
    out["gemm_8192_strong_gather_fused"] = {"ms": round(ms, 4), "TFLOP/s": round(gemm_flops() / (ms / 1e3) / 1e12, 1),
                                            "nvlink_bytes_out_per_rank": link,
                                            "nvlink_GB/s_out_per_rank": round(link / (ms / 1e3) / 1e9, 1)}
    gbuf.close()
    full = torch.empty(GEMM_M, GEMM_N, device="cuda")

    def gemm_then_nccl():
        check(tk_b200.gemm_raw(rows, GEMM_N, GEMM_K, a, GEMM_K, b, GEMM_N, c, GEMM_N))
        dist.all_gather_into_tensor(full, c)
    ms = timed(gemm_then_nccl)
    out["gemm_8192_strong_gather_nccl"] = {"ms": round(ms, 4), "TFLOP/s": round(gemm_flops() / (ms / 1e3) / 1e12, 1)}
    del a, b, c, full

    # Attention [8, 32, 4096, 128] split by batch x head (unmasked and causal), and the
    # unmasked output gathered with NCCL.
    s0, s1 = tkd.attention_slices(ATT_B, ATT_H, world, rank)
    nbh = s1 - s0
    gen.manual_seed(4)
    q = torch.randn(nbh, ATT_S, ATT_D, device="cuda", generator=gen).half()
    k = torch.randn(nbh, ATT_S, ATT_D, device="cuda", generator=gen).half()
    v = torch.randn(nbh, ATT_S, ATT_D, device="cuda", generator=gen).half()
    o = torch.empty(nbh, ATT_S, ATT_D, device="cuda")
    scale = 1.0 / math.sqrt(ATT_D)
    for causal in (False, True):
        ms = timed(lambda causal=causal: check(tk_b200.attention_raw(q, k, v, o, 1, nbh, ATT_S, ATT_D, scale, causal)))
        tf = attn_flops(causal) / (ms / 1e3) / 1e12
        out["attention_fwd_strong" + ("_causal" if causal else "")] = {
            "ms": round(ms, 4), "TFLOP/s": round(tf, 1), "frac_per_gpu": round(tf / world / burst, 4),
            "heads_per_rank": nbh}
    o_full = torch.empty(ATT_B * ATT_H, ATT_S, ATT_D, device="cuda")

    def attn_then_nccl():
        check(tk_b200.attention_raw(q, k, v, o, 1, nbh, ATT_S, ATT_D, scale, False))
        dist.all_gather_into_tensor(o_full, o)
    ms = timed(attn_then_nccl)
    out["attention_fwd_strong_gather_nccl"] = {"ms": round(ms, 4),
                                               "TFLOP/s": round(attn_flops(False) / (ms / 1e3) / 1e12, 1)}
    del q, k, v, o, o_full

    # Row ops, 1,048,576 tiles split by tile range, all four ops fused.
    t0_, t1_ = tkd.tile_range(ROW_TILES, world, rank)
    nt = t1_ - t0_
    gen.manual_seed(1)
    x = torch.randn(nt * 256, device="cuda", generator=gen) * 2
    rs = torch.empty(nt * 16, device="cuda")
    rm = torch.empty(nt * 16, device="cuda")
    sm = torch.empty(nt * 256, device="cuda")
    cs = torch.empty(nt * 256, device="cuda")
    ms = timed(lambda: check(tk_b200.row_ops_raw(x, nt, rs, rm, sm, cs)))
    nbytes = ROW_TILES * (1024 + 2 * 64 + 2 * 1024)
    gbs = nbytes / (ms / 1e3) / 1e9
    out["rowops_all4_strong"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_per_gpu": round(gbs / world / hbm, 4),
                                 "tiles_per_rank": nt}
    del x, rs, rm, sm, cs
    return out


def run_sustained(seconds: float):
    """Sustained rates under the 1 kW power cap, one GPU: each kernel back to back for
    `seconds` (events around batches of 10 calls), with nvidia-smi sampling the SM clock
    and board power meanwhile. Ours: the 8192^3 GEMM and the [8,32,4096,128] attention
    (unmasked, causal). For comparison on the same GPU, library kernels of the same
    shapes: cuBLAS FP16 x FP16 -> FP32 (torch.mm with out_dtype) and cuDNN's attention
    (torch SDPA, binary16 output). Prints one JSON line."""
    import torch
    import torch.nn.functional as F
    import tk_b200
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1)
    rows = []

    def measure(name, fn, flops, library=False):
        try:
            fn()
            torch.cuda.synchronize()
        except Exception as e:  # a library kernel this build of torch does not offer
            rows.append({"kernel": name, "unavailable": str(e).splitlines()[0][:160]})
            return
        smi = subprocess.Popen(["nvidia-smi", "--query-gpu=clocks.sm,power.draw,clocks_event_reasons.active",
                                "--format=csv,noheader,nounits", "-lms", "50", "-i",
                                str(torch.cuda.current_device())], stdout=subprocess.PIPE, text=True)
        time.sleep(0.3)
        per_call = []
        t0 = time.time()
        while time.time() - t0 < seconds:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                fn()
            e1.record()
            torch.cuda.synchronize()
            per_call.append(e0.elapsed_time(e1) / 10)
        smi.terminate()
        samples = [r.split(",") for r in smi.communicate()[0].strip().splitlines() if r.count(",") == 2]
        mhz = [float(s[0]) for s in samples]
        watts = [float(s[1]) for s in samples]
        ms = statistics.median(per_call)
        rows.append({"kernel": name, "library": library, "calls": 10 * len(per_call),
                     "first_batch_TFLOP/s": round(flops / per_call[0] / 1e9, 1),
                     "sustained_TFLOP/s": round(flops / ms / 1e9, 1), "ms_per_call": round(ms, 4),
                     "sm_mhz_median": statistics.median(mhz) if mhz else None,
                     "power_w_median": statistics.median(watts) if watts else None,
                     "reasons": sorted({s[2].strip() for s in samples})})

    def check(code):
        if code != 0:
            raise RuntimeError(f"call failed with cudaError {code}")

    n = GEMM_M
    a = (torch.rand(n, n, device="cuda", generator=gen) * 2 - 1).half()
    b = (torch.rand(n, n, device="cuda", generator=gen) * 2 - 1).half()
    c = torch.empty(n, n, device="cuda")
    measure("gemm_8192_fp16_fp32", lambda: check(tk_b200.gemm_raw(n, n, n, a, n, b, n, c, n)), gemm_flops())
    measure("cublas_gemm_8192_fp16_fp32", lambda: torch.mm(a, b, out_dtype=torch.float32), gemm_flops(), True)
    del a, b, c
    q = torch.randn(ATT_B, ATT_H, ATT_S, ATT_D, device="cuda", generator=gen).half()
    k = torch.randn(ATT_B, ATT_H, ATT_S, ATT_D, device="cuda", generator=gen).half()
    v = torch.randn(ATT_B, ATT_H, ATT_S, ATT_D, device="cuda", generator=gen).half()
    o = torch.empty(ATT_B, ATT_H, ATT_S, ATT_D, device="cuda")
    scale = 1.0 / math.sqrt(ATT_D)
    for causal in (False, True):
        tag = "_causal" if causal else ""
        measure("attention_fwd" + tag, lambda causal=causal: check(
            tk_b200.attention_raw(q, k, v, o, ATT_B, ATT_H, ATT_S, ATT_D, scale, causal)), attn_flops(causal))

        def cudnn(causal=causal):
            from torch.nn.attention import SDPBackend, sdpa_kernel
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        measure("cudnn_attention_fwd" + tag, cudnn, attn_flops(causal), True)
    print(json.dumps({"sustained": rows, "seconds_per_kernel": seconds, "status": tk_b200.device_status()}))


def workload_config(args, world):
    """The `config` object of both arms' JSON lines."""
    return {
        "workload": {"headline": "GEMM f16 8192x8192x8192 -> f32 + attention fwd [8,32,4096,128] "
                                 "unmasked + causal, per GPU",
                     "gemm": "GEMM f16 8192x8192x8192 -> f32, per GPU",
                     "attention": "attention fwd [8,32,4096,128] unmasked + causal, per GPU",
                     "rowops": f"{args.row_tiles:,} 16x16 FP32 tiles, sum+max+softmax+causal in one pass, "
                               "per GPU"}[args.workload],
        "parallelism": f"dp{world} (GEMM by M row blocks, attention by batch x head, row ops by tile range)",
        "l2": "inputs larger than L2 (126 MB): no flush needed",
        "gather": args.gather or False,
        "attention_kernel": args.attention_kernel,
    }


def main_ours(args):
    rank, world, local = init_dist()
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    wl, ms_per_step, per_kernel_ms, work_per_step, clocks, e2e_ms, h2d, d2h = run_ours(args, rank, world,
                                                                                        local)
    peaks, peak_src = load_peaks()
    traffic = load_traffic()
    timed_seconds = ms_per_step * args.steps / 1e3
    if args.workload == "rowops":
        unit, metric_scale, peak_key = "GB/s", 1e9, "hbm_gbs"
        metric = "tile row ops (sum, max, softmax, causal softmax) HBM GB/s"
        dtype = "f32"
    else:
        unit, metric_scale = "TFLOP/s", 1e12
        _, peak_key = tensor_peak(peaks, timed_seconds)
        metric = ("FP16 GEMM TFLOP/s @8192^3 + attn-fwd TFLOP/s, % of B200 peak, at 1/2/4/8 GPUs")
        dtype = "f16 in, f32 accumulate/out"
    # The hosts' copy ceiling for e2e: the step's bytes in and out, every rank at once.
    link = host_link(rank, world, wl.h2d, wl.d2h)
    link["e2e_ceiling"] = round(work_per_step / (link["ms"] / 1e3) / metric_scale, 2)
    link["e2e_ceiling_unit"] = unit
    configs = None
    multi = None
    if not args.no_configs and args.workload == "headline":
        if world == 1:
            configs = run_configs(peaks, traffic)
        else:
            multi = run_multi_gpu(rank, world, peaks)
    value = work_per_step / (ms_per_step / 1e3) / metric_scale
    e2e_value = work_per_step / (e2e_ms / 1e3) / metric_scale

    # Roofline of the dominant kernel (largest share of step time).
    dom = max(range(len(wl.call_meta)), key=lambda i: per_kernel_ms[i])
    name, work = wl.call_meta[dom]
    achieved = work / (per_kernel_ms[dom] / 1e3) / metric_scale
    peak = peaks.get(peak_key, FALLBACK_PEAKS[peak_key])
    entry = traffic.get(name, {}) if traffic else {}
    traffic_bytes = entry.get("dram_bytes_per_launch")
    if traffic_bytes is None and "dram_bytes_per_tile" in entry:
        # Captured on a smaller tile count; DRAM traffic scales with the tiles processed.
        traffic_bytes = round(entry["dram_bytes_per_tile"] * args.row_tiles)
    roofline = {"kernel": name, "bound": "hbm" if unit == "GB/s" else "tensor", "achieved": round(achieved, 1),
                "peak": peak, "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic_bytes,
                "peak_source": f"{peak_src} {peak_key} (timed region {timed_seconds:.2f} s)"}
    if unit == "TFLOP/s":
        roofline["frac_of_sustained"] = round(
            achieved / peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]), 4)
    components = {}
    for (cname, cwork), ms in zip(wl.call_meta, per_kernel_ms):
        rate = cwork / (ms / 1e3) / metric_scale
        components[cname] = {"ms": round(ms, 4), unit: round(rate, 1), "frac": round(rate / peak, 4)}

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and args.workload != "rowops":
            threads = min(os.cpu_count() or 1, 64)
            res = cpu_baseline(threads, args.workload)
            if res is not None:
                tflops, kind, sample, secs, legs = res
                cpu = {"value": tflops, "unit": unit, "cores": threads, "kind": kind, "legs": legs,
                       "sample": f"{sample}; {secs:.1f} s wall with {threads} threads, scaled to the step's "
                                 "FLOP mix"}
        config = workload_config(args, world)
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded, on device)",
            "config": config, "roofline": roofline, "components": components,
            "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": wl.launches_per_step * args.steps,
            "clocks": clocks, "cpu_baseline": cpu, "host_link": link,
        }
        if configs is not None:
            line["configs"] = configs
        if multi is not None:
            line["multi_gpu"] = multi
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        if wl.gbuf is not None:
            wl.gbuf.close()  # collective
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------
# Reference arm
# ---------------------------------------------------------------------------------

def main_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if args.workload == "rowops":
        unit = "GB/s"
        metric = "tile row ops (sum, max, softmax, causal softmax) HBM GB/s"
    else:
        unit = "TFLOP/s"
        metric = "FP16 GEMM TFLOP/s @8192^3 + attn-fwd TFLOP/s, % of B200 peak, at 1/2/4/8 GPUs"
    values, kinds, samples, secs, legs = [], set(), "", [], {}
    for i in range(args.warmup + args.steps):
        if args.workload == "rowops":
            import numpy as np

            import oracle
            n = 4096 * threads
            tiles = oracle.gen_normal_f32(1, 2.0, n * 256)
            t0 = time.perf_counter()
            per = n // threads

            def work(j):
                sl = tiles[j * per * 256:(j + 1) * per * 256]
                oracle.tile_row_reduce(sl, "sum")
                oracle.tile_row_reduce(sl, "max")
                oracle.tile_row_softmax_f64(sl, False)
                oracle.tile_row_softmax_f64(sl, True)
            ts = [threading.Thread(target=work, args=(j,)) for j in range(threads)]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            dt = time.perf_counter() - t0
            val = (n * 1024 * 3 + n * 128) / dt / 1e9
            kind, sample = "port", f"{n} tiles (restated row-tree and FP64 softmax oracles)"
            legs = {"rowops": "port"}
        else:
            # The cpu_baseline leg's sample: about 1.5 s per step with all host threads.
            val, kind, sample, dt, legs = cpu_baseline(threads, args.workload)
        if i >= args.warmup:
            values.append(val)
            kinds.add(kind)
            samples = sample
            secs.append(dt)
    value = statistics.median(values)
    kind = "reference" if kinds == {"reference"} else "port"
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.median(secs) * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64 (host oracle)",
        "data": "synthetic (seeded)",
        "config": dict(workload_config(args, world), sample_per_step=samples),
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": kind, "legs": legs,
                         "sample": samples},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["headline", "gemm", "attention", "rowops"], default="headline")
    ap.add_argument("--gather", nargs="?", const="fused", default=None, choices=["fused", "nccl"],
                    help="gather each step's outputs on every rank: 'fused' (default) stores the GEMM's C "
                         "into every rank's buffer from the GEMM epilogue and all-gathers the attention "
                         "outputs with NCCL; 'nccl' all-gathers every output with NCCL after its kernel")
    ap.add_argument("--row-tiles", type=int, default=ROW_TILES,
                    help="tiles per GPU of the rowops workload (default 1,048,576; inputs stay larger than L2 "
                         "above 126,000)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attention-kernel", choices=["cta1", "pair"], default="cta1",
                    help="head_dim 128 attention kernel: single-CTA (default) or CTA pair (tcgen05 cta_group::2)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-configuration (N = 1) and multi-GPU (N > 1) measurements")
    ap.add_argument("--sustained", type=float, default=0.0, metavar="SECONDS",
                    help="instead of the benchmark line: sustained rates under the power cap (one GPU), each "
                         "kernel back to back for SECONDS, with cuBLAS / cuDNN kernels of the same shapes "
                         "measured beside ours")
    args = ap.parse_args()
    if args.sustained > 0:
        if args.gpus != 1:
            raise SystemExit("--sustained runs on one GPU")
        run_sustained(args.sustained)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        main_reference(args)
    else:
        main_ours(args)


if __name__ == "__main__":
    main()
