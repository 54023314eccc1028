"""Per-call latency of the public entry points, measured by a C++ caller
(tests/latency/call_latency.cu) with the reference benches' own methods: GEMM
best-of-5 single calls at square sizes 256..4096 (bench/gemm_throughput.cu:94-120),
one-tile attention as the median of 4 rounds of 2048 back-to-back calls
(bench/attention_throughput.cu:128-165, 206-233). When oracle/_ref/libtk_legacy.so
exists (the reference's kernels as compute_75 PTX), the same caller measures it on
the same GPU. Run with ``-s`` to see the table."""

import json
import os
import subprocess

import pytest

import oracle
import tk_b200

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_call_latency(tmp_path):
    exe = tmp_path / "call_latency"
    lib_dir = os.path.dirname(tk_b200.LIB_PATH)
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "latency", "call_latency.cu"), "-o", str(exe), "-L", lib_dir,
                    "-ltk_b200", f"-Xlinker=-rpath={lib_dir}", "-ldl"], check=True)
    cmd = [str(exe)]
    if os.path.exists(oracle.LEGACY_SO):
        cmd.append(oracle.LEGACY_SO)
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    rows = [json.loads(line) for line in out.stdout.splitlines() if line.startswith("{")]
    table = {}
    for r in rows:
        table.setdefault(r["call"], {})[r["impl"]] = (r["us"], r["host_us"])
    print("\nper-call latency, us (host time inside the call in brackets):")
    for call, by_impl in table.items():
        print(f"  {call:24s} " + "  ".join(f"{k} {v[0]:9.2f} ({v[1]:6.2f})" for k, v in sorted(by_impl.items())))
    assert all(r["us"] > 0 for r in rows)
    assert {"gemm_256", "gemm_4096", "attention_16x16", "attention_16x16_causal"} <= set(table)
