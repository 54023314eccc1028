"""The allocation-free row-statistics GEMM, for callers that cannot allocate.

Some callers of this library own all device memory themselves (a custom arena
allocator, a host application that forbids allocation once it is running, or a
latency-critical path where an allocation could block), so they cannot let the
library call cudaMalloc or the stream-ordered allocator for scratch. For them
tk_gemm_f16_f16_f32_nn_rowstats_noalloc keeps its per-tile partials in a fixed
array compiled into the library. This test calls it through the C ABI twice in a
row, with different shapes, and checks that each call returns exactly what the
allocating entry point tk_gemm_f16_f16_f32_nn_rowstats returns (the same kernel
and reduction order, so the bits must agree): on single-CTA tiles, on CTA pairs,
and on a problem that needs exactly as many partials as the array holds. A
problem one tile larger is refused without touching any output, and a call made
first in a fresh process leaves the library's scratch pool uncreated (nothing
was allocated), while the allocating entry point does create it.

It lives in its own file named so that pytest collects it last, and it makes no
assumption about what ran before it in the same process.
"""

import numpy as np
import pytest
import torch

import oracle
import tk_b200

pytestmark = pytest.mark.gpu


def to_device(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.float16).cuda()


def both_entry_points(m, n, k, seed, oracle_rows=None):
    a, b = oracle.gen_gemm_uniform(seed, m, n, k, k, n)
    da, db = to_device(a), to_device(b)
    stream = torch.cuda.current_stream().cuda_stream
    lib = tk_b200.lib()
    outs = []
    for fn in (lib.tk_gemm_f16_f16_f32_nn_rowstats, lib.tk_gemm_f16_f16_f32_nn_rowstats_noalloc):
        c = torch.full((m, n), float("nan"), device="cuda")
        mx = torch.full((m,), float("nan"), device="cuda")
        sm = torch.full((m,), float("nan"), device="cuda")
        assert fn(m, n, k, da.data_ptr(), k, db.data_ptr(), n, c.data_ptr(), n, mx.data_ptr(),
                  sm.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        outs.append((c.cpu().numpy(), mx.cpu().numpy(), sm.cpu().numpy()))
    (c0, mx0, sm0), (c1, mx1, sm1) = outs
    # Same results as the allocating entry point, bit for bit.
    assert np.array_equal(c1.view(np.uint32), c0.view(np.uint32))
    assert np.array_equal(mx1.view(np.uint32), mx0.view(np.uint32))
    assert np.array_equal(sm1.view(np.uint32), sm0.view(np.uint32))
    # And C within the GEMM error model against the FP64 oracle on a few rows.
    rows = [0, m // 2, m - 1] if oracle_rows is None else oracle_rows
    for r in rows:
        ref, s = oracle.gemm_ref(m, n, k, a, k, b, n, row_begin=r, row_end=r + 1)
        assert oracle.gemm_check(k, c1[r:r + 1], ref, s, n, n)[0] == 0
    want_max, want_sum = oracle.matrix_row_stats(c1, m, n, n)
    assert np.array_equal(mx1.view(np.uint32), want_max.view(np.uint32))
    assert np.array_equal(sm1.view(np.uint32), want_sum.view(np.uint32))


def test_no_alloc_matches_allocating_entry_point_twice_in_a_row():
    # First call: a larger problem fills more of the shared scratch ...
    both_entry_points(1024, 4096, 256, seed=21)
    # ... second call: a smaller one must not see anything left by the first.
    both_entry_points(384, 1040, 128, seed=22)
    assert tk_b200.device_status() == 0


def test_no_alloc_on_cta_pairs():
    # 1024 x 4096 has 64 tiles of 256 x 256, below the 74 that make the library
    # choose CTA pairs on its own: force the pair kernel, whose epilogue writes the
    # partials from both CTAs of each tile.
    lib = tk_b200.lib()
    old = lib.tk_gemm_set_cta_group(2)
    try:
        both_entry_points(1024, 4096, 192, seed=23)
    finally:
        lib.tk_gemm_set_cta_group(old)
    assert tk_b200.device_status() == 0


def test_no_alloc_at_its_exact_limit():
    # m * ceil(n / 256) == TK_GEMM_ROWSTATS_NOALLOC_MAX_PARTIALS: accepted, every
    # slot of the array used once.
    m, n = 4096, 32768
    assert m * (n // 256) == 1 << 19
    both_entry_points(m, n, 64, seed=24, oracle_rows=[0, m - 1])
    assert tk_b200.device_status() == 0


_FRESH_PROCESS = r"""
import sys
sys.path[:0] = sys.argv[1:3]
import numpy as np, torch
import oracle, tk_b200
torch.cuda.set_device(0)
m, n, k = 512, 1024, 128
a, b = oracle.gen_gemm_uniform(25, m, n, k, k, n)
da = torch.from_numpy(a.view(np.int16).copy()).view(torch.float16).cuda()
db = torch.from_numpy(b.view(np.int16).copy()).view(torch.float16).cuda()
c = torch.empty(m, n, device="cuda"); mx = torch.empty(m, device="cuda"); sm = torch.empty(m, device="cuda")
lib = tk_b200.lib()
args = (m, n, k, da.data_ptr(), k, db.data_ptr(), n, c.data_ptr(), n, mx.data_ptr(), sm.data_ptr(), None)
assert lib.tk_gemm_f16_f16_f32_nn_rowstats_noalloc(*args) == 0
torch.cuda.synchronize()
print("after_noalloc", *tk_b200.scratch_pool_bytes(0))
assert lib.tk_gemm_f16_f16_f32_nn_rowstats(*args) == 0
torch.cuda.synchronize()
print("after_alloc", *tk_b200.scratch_pool_bytes(0))
print("status", tk_b200.device_status())
"""


def test_no_alloc_allocates_nothing():
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    out = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, root,
                          os.path.join(root, "thunderkittens-sm7x_b200")],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    vals = {line.split()[0]: [int(x) for x in line.split()[1:]] for line in out.stdout.splitlines() if line}
    # The no-allocation entry point ran first: the library's pool does not exist yet.
    assert vals["after_noalloc"] == [0, 0]
    # The allocating entry point then took (and returned) its pairs from the pool.
    reserved, used = vals["after_alloc"]
    assert reserved >= 512 * 4 * 8 and used == 0
    assert vals["status"] == [0]


def test_no_alloc_rejects_problems_larger_than_its_scratch():
    lib = tk_b200.lib()
    limit = 1 << 19  # TK_GEMM_ROWSTATS_NOALLOC_MAX_PARTIALS
    m = 8192
    n = (limit // m + 1) * 256  # one 256-column tile more than fits
    row_max = torch.full((m,), 3.0, device="cuda")
    row_sum = torch.full((m,), 4.0, device="cuda")
    fake = 1 << 20  # aligned A, B, C addresses that are never dereferenced: the call refuses first
    code = lib.tk_gemm_f16_f16_f32_nn_rowstats_noalloc(m, n, 64, fake, 64, fake, n, fake, n,
                                                       row_max.data_ptr(), row_sum.data_ptr(), None)
    assert code == tk_b200.CUDA_ERROR_NOT_SUPPORTED
    torch.cuda.synchronize()
    assert torch.all(row_max == 3.0) and torch.all(row_sum == 4.0)
