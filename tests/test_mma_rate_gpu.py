"""Measured tcgen05.mma rates behind the attention kernel's roofline
(tests/microbench/mma_rate.cu): cycles per M = 128 kind::f16 MMA issued back to
back, with shared-memory B operands reused by consecutive groups or fresh, as in a
real kernel. Run with ``-s`` to see the table."""

import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_mma_rates(tmp_path):
    exe = tmp_path / "mma_rate"
    subprocess.run(["nvcc", "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", os.path.join(ROOT, "thunderkittens-sm7x_b200", "csrc"), "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "microbench", "mma_rate.cu"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    rows = {r["case"]: r for r in (json.loads(line) for line in out.stdout.splitlines() if line.startswith("{"))}
    print("\ncycles per tcgen05.mma (M = 128, K = 16):")
    for name, r in rows.items():
        print(f"  {name:24s} {r['cycles_per_mma']:7.1f}  (dense-rate ideal {r['ideal']})")
    assert len(rows) == 13 and all(r["cycles_per_mma"] > 0 for r in rows.values())
    # No case can beat the dense tensor rate.
    assert all(r["cycles_per_mma"] >= 0.95 * r["ideal"] for r in rows.values())
