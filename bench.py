"""Benchmark of the ThunderKittens-SM7x hot path on B200 (one process per GPU).

Headline step (per GPU, weak scaling): one FP16 x FP16 -> FP32 GEMM of
8192 x 8192 x 8192 (this rank's 8192-row block of an (8192 * N)-row A, with B
replicated), one attention forward over [8, 32, 4096, 128] unmasked and one causal
(this rank's batch x head shard). value = all FLOPs of all ranks / max-over-ranks
device time, in TFLOP/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload headline|gemm|attention|rowops] [--gather]

Timing: K steps between two CUDA events on the launching stream, a barrier and
torch.cuda.synchronize() on both sides, the max over ranks. Inputs are larger than
L2 (126 MB), so consecutive steps cannot be served from cache. e2e repeats the
step through the same C ABI with host buffers: pinned host -> device copies of the
step's inputs and device -> host copies of its outputs inside the timed region.

--impl reference times the reference's CPU implementation of the path (its FP64
host GEMM oracle compiled from its sources, oracle/_ref; the generalised FP64
attention oracle) on bounded row samples with all host threads, on rank 0 only.
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
    fused = args.gather == "fused"
    wl = Workload(args.workload, rank, world, args.row_tiles, fused_gather=fused)
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


def cpu_baseline(threads: int, workload: str, gemm_rows: int = 32, attn_rows: int = 1024):
    """Returns (TFLOP/s over the sampled work, kind, description, CPU seconds) for the
    step's FLOP mix. The defaults give about 10 s of CPU work."""
    parts = []
    kind = "port"
    if workload in ("headline", "gemm"):
        f, dt, kind, desc = cpu_sample_gemm(threads, rows_per_thread=gemm_rows)
        parts.append((f, dt, desc))
    if workload in ("headline", "attention"):
        f, dt, desc = cpu_sample_attention(threads, min(attn_rows, ATT_S), False)
        parts.append((f, dt, desc))
    if not parts:
        return None
    # Time the sampled work of each kernel and scale to the step's FLOP mix.
    step_mix = {"headline": [gemm_flops(), attn_flops(False) + attn_flops(True)],
                "gemm": [gemm_flops()], "attention": [attn_flops(False) + attn_flops(True)]}[workload]
    step_seconds = sum(mix / (f / dt) for mix, (f, dt, _) in zip(step_mix, parts))
    tflops = sum(step_mix) / step_seconds / 1e12
    sample = "; ".join(d for _, _, d in parts)
    return tflops, kind, sample, sum(dt for _, dt, _ in parts)


def main_ours(args):
    rank, world, local = init_dist()
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    wl, ms_per_step, per_kernel_ms, work_per_step, clocks, e2e_ms, h2d, d2h = run_ours(args, rank, world,
                                                                                        local)
    peaks, peak_src = load_peaks()
    traffic = load_traffic()
    if args.workload == "rowops":
        unit, metric_scale, peak_key = "GB/s", 1e9, "hbm_gbs"
        metric = "tile row ops (sum, max, softmax, causal softmax) HBM GB/s"
        dtype = "f32"
    else:
        unit, metric_scale, peak_key = "TFLOP/s", 1e12, "bf16_tflops_sustained"
        metric = ("FP16 GEMM TFLOP/s @8192^3 + attn-fwd TFLOP/s, % of B200 peak, at 1/2/4/8 GPUs")
        dtype = "f16 in, f32 accumulate/out"
    value = work_per_step / (ms_per_step / 1e3) / metric_scale
    e2e_value = work_per_step / (e2e_ms / 1e3) / metric_scale

    # Roofline of the dominant kernel (largest share of step time).
    dom = max(range(len(wl.calls)), key=lambda i: per_kernel_ms[i])
    name, _, work, _ = wl.calls[dom]
    achieved = work / (per_kernel_ms[dom] / 1e3) / metric_scale
    peak = peaks.get(peak_key, FALLBACK_PEAKS[peak_key])
    entry = traffic.get(name, {}) if traffic else {}
    traffic_bytes = entry.get("dram_bytes_per_launch")
    if traffic_bytes is None and "dram_bytes_per_tile" in entry:
        # Captured on a smaller tile count; DRAM traffic scales with the tiles processed.
        traffic_bytes = round(entry["dram_bytes_per_tile"] * args.row_tiles)
    roofline = {"kernel": name, "bound": "hbm" if unit == "GB/s" else "tensor", "achieved": round(achieved, 1),
                "peak": peak, "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic_bytes,
                "peak_source": f"{peak_src} {peak_key}"}
    if unit == "TFLOP/s":
        roofline["frac_of_burst"] = round(achieved / peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]), 4)
    components = {}
    for (cname, _, cwork, _), ms in zip(wl.calls, per_kernel_ms):
        rate = cwork / (ms / 1e3) / metric_scale
        components[cname] = {"ms": round(ms, 4), unit: round(rate, 1), "frac": round(rate / peak, 4)}

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and args.workload != "rowops":
            threads = min(os.cpu_count() or 1, 64)
            res = cpu_baseline(threads, args.workload)
            if res is not None:
                tflops, kind, sample, secs = res
                cpu = {"value": tflops, "unit": unit, "cores": threads, "kind": kind,
                       "sample": f"{sample}; {secs:.1f} s of CPU time, scaled to the step's FLOP mix"}
        config = {
            "workload": {"headline": "GEMM f16 8192x8192x8192 -> f32 + attention fwd [8,32,4096,128] "
                                     "unmasked + causal, per GPU",
                         "gemm": "GEMM f16 8192x8192x8192 -> f32, per GPU",
                         "attention": "attention fwd [8,32,4096,128] unmasked + causal, per GPU",
                         "rowops": f"{args.row_tiles:,} 16x16 FP32 tiles, sum+max+softmax+causal in one pass, "
                                   "per GPU"}[args.workload],
            "parallelism": f"dp{world} (GEMM by M row blocks, attention by batch x head, row ops by tile range)",
            "l2": "inputs larger than L2 (126 MB): no flush needed",
            "gather": args.gather or False,
        }
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded, on device)",
            "config": config, "roofline": roofline, "components": components,
            "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": sum(c[3] for c in wl.calls) * args.steps,
            "clocks": clocks, "cpu_baseline": cpu,
        }
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
    values, kinds, samples, secs = [], set(), "", []
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
        else:
            # About 1.5 s of CPU work per step, so the whole run stays within minutes.
            val, kind, sample, dt = cpu_baseline(threads, args.workload, gemm_rows=4, attn_rows=128)
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
        "config": {"workload": args.workload, "sample_per_step": samples},
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": kind, "sample": samples},
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
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        main_reference(args)
    else:
        main_ours(args)


if __name__ == "__main__":
    main()
