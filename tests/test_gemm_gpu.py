"""GEMM on the GPU through the C ABI, against the CPU oracle.

Exact-domain cases must equal the FP64 reference bit for bit; model-domain
cases must stay within error_bound(k, S) (tests/numerical_bounds.hpp:9-28, and
its uncapped extension for K > 1024); C padding must keep its sentinel
(tests/gemm_correctness.cu:147-155, tests/gemm_differential.cu:412-418)."""

import numpy as np
import pytest
import torch

import oracle
import tk_b200
from oracle import fixtures as fx
from cuda_util import cudart, dev, host, seed_stale_error

pytestmark = pytest.mark.gpu

NAN_BITS = 0x7FC00000  # tests/gemm_differential.cu:22


def run_gemm(m, n, k, a, lda, b, ldb, ldc, sentinel=None, cta_group=0):
    fill = np.uint32(NAN_BITS).view(np.float32) if sentinel is None else sentinel
    c_host = np.full((m, ldc), fill, dtype=np.float32)
    da, db, dc = dev(a), dev(b), dev(c_host)
    prev = tk_b200.set_gemm_cta_group(cta_group)
    try:
        code = tk_b200.gemm_raw(m, n, k, da, lda, db, ldb, dc, ldc)
    finally:
        tk_b200.set_gemm_cta_group(prev)
    assert code == 0
    return host(dc)


def padding_intact(c, n, sentinel_bits):
    return np.all(c[:, n:].view(np.uint32) == sentinel_bits)


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("case", fx.DIFFERENTIAL_EXACT_CASES, ids=lambda c: c[0])
def test_differential_exact(case, cta_group):
    name, m, n, k, lda, ldb, ldc, pattern = case
    a, b = fx.differential_inputs(m, n, k, lda, ldb, pattern)
    r, _ = oracle.gemm_ref(m, n, k, a, lda, b, ldb)
    c = run_gemm(m, n, k, a, lda, b, ldb, ldc, cta_group=cta_group)
    assert np.array_equal(c[:, :n].astype(np.float64), r)
    assert padding_intact(c, n, NAN_BITS)


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("case", fx.DIFFERENTIAL_MODEL_CASES, ids=lambda c: c[0])
def test_differential_model(case, cta_group):
    name, m, n, k, lda, ldb, ldc, pattern = case
    a, b = fx.differential_inputs(m, n, k, lda, ldb, pattern)
    r, s = oracle.gemm_ref(m, n, k, a, lda, b, ldb)
    c = run_gemm(m, n, k, a, lda, b, ldb, ldc, cta_group=cta_group)
    fails, max_abs, ratio = oracle.gemm_check(k, c, r, s, n, ldc, NAN_BITS, check_padding=True)
    assert fails == 0, (max_abs, ratio)
    bound = np.vectorize(lambda x: oracle.error_bound(k, x))(s)  # the reference's own (K <= 1024) bound
    assert np.all(np.abs(c[:, :n] - r) <= bound)


@pytest.mark.parametrize("case", fx.CORRECTNESS_CASES, ids=lambda c: c[0])
def test_correctness_roster(case):
    """tests/gemm_correctness.cu:434-449: strided, odd leading dimensions, small/large
    tiles and the grid-y boundary case with 8,388,608 rows."""
    name, m, n, k, lda, ldb, ldc, pattern, seed, exact = case
    a, b = fx.correctness_inputs(m, n, k, lda, ldb, pattern, seed)
    sentinel = fx.CORR_SENTINEL
    c = run_gemm(m, n, k, a, lda, b, ldb, ldc, sentinel=sentinel)
    assert np.all(c[:, n:] == sentinel)
    if pattern == fx.CORR_IDENTITY_RIGHT:
        assert np.array_equal(c[:, :n], oracle.f16_bits_to_f32(a[:, :n]))
        return
    r, _ = oracle.gemm_ref(m, n, k, a, lda, b, ldb)
    ref = r.astype(np.float32)
    if exact:
        assert np.array_equal(c[:, :n], ref)
    else:
        assert np.all(np.abs(c[:, :n] - ref) <= 2e-3 + 2e-3 * np.abs(ref))


def test_gemm_256_seed0():
    """The 256^3 configuration: uniform [-1, 1] from std::mt19937(0), A then B."""
    a, b = oracle.gen_gemm_uniform(0, 256, 256, 256, 256, 256)
    r, s = oracle.gemm_ref(256, 256, 256, a, 256, b, 256)
    for g in (1, 2):
        c = run_gemm(256, 256, 256, a, 256, b, 256, 256, cta_group=g)
        assert oracle.gemm_check(256, c, r, s, 256, 256)[0] == 0
        assert np.all(np.abs(c - r) <= 2e-3 + 2e-3 * np.abs(r))


def test_misaligned_pointers():
    """2-byte aligned A/B (repacked for TMA) and 4-byte aligned C (scalar stores)."""
    m, n, k = 48, 80, 96
    a, b = oracle.gen_gemm_uniform(11, m, n, k, k, n)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    da = dev(np.concatenate([[0], a.reshape(-1)]).astype(np.uint16))
    db = dev(np.concatenate([[0], b.reshape(-1)]).astype(np.uint16))
    dc = torch.full((m * n + 1,), float("nan"), device="cuda")
    assert tk_b200.gemm_raw(m, n, k, da.data_ptr() + 2, k, db.data_ptr() + 2, n, dc.data_ptr() + 4, n) == 0
    c = host(dc)[1:].reshape(m, n)
    assert oracle.gemm_check(k, c, r, s, n, n)[0] == 0
    assert np.isnan(host(dc)[0])


def test_rowstats_bit_exact_on_gpu_output():
    """Fused row max / sum equal the fixed-order reduction of the GPU's own C."""
    for (m, n, k, g) in ((384, 1040, 256, 1), (512, 4096, 128, 2), (16, 16, 16, 1), (272, 784, 64, 2)):
        a, b = oracle.gen_gemm_uniform(m + n, m, n, k, k, n)
        da, db = dev(a), dev(b)
        prev = tk_b200.set_gemm_cta_group(g)
        try:
            c, mx, sm = tk_b200.gemm_rowstats(da, db)
        finally:
            tk_b200.set_gemm_cta_group(prev)
        c = host(c)
        r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
        assert oracle.gemm_check(k, c, r, s, n, n)[0] == 0
        want_max, want_sum = oracle.matrix_row_stats(c, m, n, n)
        assert np.array_equal(host(mx).view(np.uint32), want_max.view(np.uint32)), (m, n, k, g)
        assert np.array_equal(host(sm).view(np.uint32), want_sum.view(np.uint32)), (m, n, k, g)


def sample_rows(m, count, seed=0):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, count)]))


def check_rows(m, n, k, a, lda, b, ldb, c, ldc, rows):
    for row in rows:
        r, s = oracle.gemm_ref(m, n, k, a, lda, b, ldb, row_begin=int(row), row_end=int(row) + 1)
        fails, max_abs, ratio = oracle.gemm_check(k, c[row:row + 1], r, s, n, ldc)
        assert fails == 0, (row, max_abs, ratio)


def test_square_8192_sampled_rows():
    m = n = k = 8192
    a, b = oracle.gen_gemm_uniform(2, m, n, k, k, n)
    da, db = dev(a), dev(b)
    c = host(tk_b200.gemm(da, db))
    check_rows(m, n, k, a, k, b, n, c, n, sample_rows(m, 30))
    _, mx, sm = tk_b200.gemm_rowstats(da, db)
    want_max, want_sum = oracle.matrix_row_stats(c, m, n, n)
    assert np.array_equal(host(mx).view(np.uint32), want_max.view(np.uint32))
    assert np.array_equal(host(sm).view(np.uint32), want_sum.view(np.uint32))


def test_padded_16384x4096x14336():
    m, n, k, lda, ldb, ldc = 16384, 4096, 14336, 14400, 4128, 4128
    pad_half = int(fx.value_from_q(7).reshape(-1)[0])  # 7/8: reading padding would corrupt results
    a, b = oracle.gen_gemm_normal(3, 0.02, m, n, k, lda, ldb, pad_bits=pad_half)
    sentinel = np.float32(-123456.0)
    c = run_gemm(m, n, k, a, lda, b, ldb, ldc, sentinel=sentinel)
    assert np.all(c[:, n:] == sentinel)
    check_rows(m, n, k, a, lda, b, ldb, c, ldc, sample_rows(m, 12))


def test_decode_16x4096x4096():
    m, n, k = 16, 4096, 4096
    a, b = oracle.gen_gemm_normal(3, 0.02, m, n, k, k, n)
    c = run_gemm(m, n, k, a, k, b, n, n)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    assert oracle.gemm_check(k, c, r, s, n, n)[0] == 0


@pytest.mark.parametrize("m,n,k,ldc,cta_group", [(48, 784, 2048, 787, 0), (304, 512, 4096, 512, 1),
                                                 (304, 512, 4096, 520, 2), (16, 4096, 4096, 4096, 0)],
                         ids=["ragged_n_scalar_c", "pairs_off", "cta_pairs", "decode"])
def test_split_k_in_kernel_reduction(m, n, k, ldc, cta_group):
    """Split-K shapes (few output tiles, long K): the partials of a tile's K splits
    are summed in split order, inside the tile's cluster (up to 8 splits on single
    CTAs) or by a second kernel. Results within the error bound, C padding untouched,
    and bit-identical across two runs (the order does not depend on timing)."""
    a, b = oracle.gen_gemm_normal(5, 0.02, m, n, k, k, n)
    sentinel = np.float32(-7.0)
    c1 = run_gemm(m, n, k, a, k, b, n, ldc, sentinel=sentinel, cta_group=cta_group)
    c2 = run_gemm(m, n, k, a, k, b, n, ldc, sentinel=sentinel, cta_group=cta_group)
    assert np.array_equal(c1.view(np.uint32), c2.view(np.uint32))
    assert np.all(c1[:, n:] == sentinel)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    assert oracle.gemm_check(k, np.ascontiguousarray(c1[:, :n]), r, s, n, n)[0] == 0
    assert tk_b200.device_status() == 0


@pytest.mark.parametrize("m,n,k,ldc", [(16, 4096, 4096, 4096), (48, 784, 2048, 787), (512, 512, 512, 512),
                                       (1024, 1024, 1024, 1032), (208, 1040, 1024, 1040)],
                         ids=["decode", "ragged_scalar_c_128_cols", "512_128_cols", "1024_4_splits_ldc",
                              "ragged_rows_cols_128_cols"])
def test_split_k_cluster_reduction_matches_kernel(m, n, k, ldc):
    """The in-cluster split-K reduction (the K splits of a tile form a cluster and sum
    their partials over distributed shared memory) and the separate reduction kernel
    add the same partials in the same order: bit-identical C, padding untouched. The
    shapes cover 256- and 128-column tiles."""
    a, b = oracle.gen_gemm_normal(7, 0.02, m, n, k, k, n)
    sentinel = np.float32(-5.0)
    prev = tk_b200.set_gemm_splitk_reduce(1)
    try:
        c_kernel = run_gemm(m, n, k, a, k, b, n, ldc, sentinel=sentinel)
        tk_b200.set_gemm_splitk_reduce(0)
        c_cluster = run_gemm(m, n, k, a, k, b, n, ldc, sentinel=sentinel)
    finally:
        tk_b200.set_gemm_splitk_reduce(prev)
    assert np.array_equal(c_cluster.view(np.uint32), c_kernel.view(np.uint32))
    assert np.all(c_cluster[:, n:] == sentinel)
    check_rows(m, n, k, a, k, b, n, c_cluster, ldc, sample_rows(m, 16))
    assert tk_b200.device_status() == 0


def test_error_state_contract():
    rt = cudart()
    a = torch.zeros((16, 16), dtype=torch.float16, device="cuda")
    c = torch.full((16, 16), 3.0, device="cuda")
    torch.cuda.synchronize()
    code = seed_stale_error()
    assert tk_b200.gemm_raw(16, 16, 17, a, 16, a, 16, c, 16) == tk_b200.CUDA_ERROR_INVALID_VALUE
    assert rt.cudaPeekAtLastError() == code
    assert rt.cudaGetLastError() == code and rt.cudaPeekAtLastError() == 0
    torch.cuda.synchronize()
    assert torch.all(c == 3.0)
    seed_stale_error()
    assert tk_b200.gemm_raw(16, 16, 16, a, 16, a, 16, c, 16) == 0
    assert rt.cudaPeekAtLastError() == 0
    torch.cuda.synchronize()
    assert torch.all(c == 0.0)
    assert tk_b200.device_status() == 0


@pytest.mark.parametrize("m,n,k,ldc,cta_group", [(512, 1024, 2048, 1024, 0), (256, 784, 512, 790, 1),
                                                 (768, 512, 1024, 520, 2)],
                         ids=["vec", "scalar_ldc", "cta_pairs"])
def test_gather_epilogue_two_local_buffers(m, n, k, ldc, cta_group):
    """tk_gemm_f16_f16_f32_nn_gather on one GPU with two local buffers standing in for
    two ranks: the call for rank r stores its m rows at rows [r m, r m + m) of both
    buffers. Every block within the error bound, padding and the other rank's rows
    untouched by a call, and the two buffers bit-identical."""
    blocks = [oracle.gen_gemm_normal(100 + r, 0.02, m, n, k, k, n) for r in range(2)]
    b = blocks[0][1]
    sentinel = np.float32(-3.0)
    bufs = [torch.full((2 * m, ldc), float(sentinel), device="cuda") for _ in range(2)]
    ptrs = [t.data_ptr() for t in bufs]
    db = dev(b)
    prev = tk_b200.set_gemm_cta_group(cta_group)
    try:
        for r in range(2):
            assert tk_b200.gemm_gather_raw(m, n, k, dev(blocks[r][0]), k, db, n, ptrs, r, ldc) == 0
            if r == 0:
                first = host(bufs[0])
                assert np.all(first[m:] == sentinel)  # rank 1's rows not written by rank 0's call
    finally:
        tk_b200.set_gemm_cta_group(prev)
    got = [host(t) for t in bufs]
    assert np.array_equal(got[0].view(np.uint32), got[1].view(np.uint32))
    assert np.all(got[0][:, n:] == sentinel)
    for r in range(2):
        ref, sabs = oracle.gemm_ref(m, n, k, blocks[r][0], k, b, n)
        part = np.ascontiguousarray(got[0][r * m:(r + 1) * m, :n])
        assert oracle.gemm_check(k, part, ref, sabs, n, n)[0] == 0
    assert tk_b200.device_status() == 0


def test_gather_invalid_arguments():
    a = torch.zeros((16, 16), dtype=torch.float16, device="cuda")
    c = torch.zeros((32, 16), device="cuda")
    p = [c.data_ptr(), c.data_ptr()]
    bad = tk_b200.CUDA_ERROR_INVALID_VALUE
    assert tk_b200.gemm_gather_raw(16, 16, 16, a, 16, a, 16, p, 2, 16) == bad   # rank out of range
    assert tk_b200.gemm_gather_raw(16, 16, 16, a, 16, a, 16, p[:1] * 9, 0, 16) == bad  # more than 8 ranks
    assert tk_b200.gemm_gather_raw(16, 16, 16, a, 16, a, 16, [c.data_ptr(), 0], 0, 16) == bad  # null buffer
    assert tk_b200.gemm_gather_raw(16, 16, 16, a, 16, a, 16, p, 0, 8) == bad   # ldc < n
    assert tk_b200.gemm_gather_raw(16, 16, 16, a, 16, a, 16, p, 1, 16) == 0


@pytest.mark.parametrize("m,n,k,lda,ldb,ldc", [
    (16, 16, 16, 16, 16, 16), (16, 4096, 4096, 4096, 4096, 4096), (32, 784, 2048, 2056, 792, 787),
    (48, 1040, 1024, 1024, 1040, 1044), (64, 20000, 96, 96, 20000, 20000), (64, 4096, 14336, 14400, 4128, 4128),
    (16, 48, 8192, 8192, 48, 48)],
    ids=["one_tile", "decode", "ragged_padded", "48_rows", "wide_short_k", "64_rows_long_k", "narrow_long_k"])
def test_small_m_operand_swapped_kernel(m, n, k, lda, ldb, ldc):
    """M <= 64 runs on the operand-swapped kernel (C^T = B^T A^T: the rows of A are the
    MMA's N). Within the error bound, C padding untouched, bit-identical over two runs and
    between the two split-K reduction forms (in the cluster / by the second kernel)."""
    a, b = oracle.gen_gemm_normal(11, 0.02, m, n, k, lda, ldb)
    sentinel = np.float32(-3.0)
    prev = tk_b200.set_gemm_splitk_reduce(0)
    try:
        c0 = run_gemm(m, n, k, a, lda, b, ldb, ldc, sentinel=sentinel)
        c0b = run_gemm(m, n, k, a, lda, b, ldb, ldc, sentinel=sentinel)
        tk_b200.set_gemm_splitk_reduce(1)
        c1 = run_gemm(m, n, k, a, lda, b, ldb, ldc, sentinel=sentinel)
    finally:
        tk_b200.set_gemm_splitk_reduce(prev)
    assert np.array_equal(c0.view(np.uint32), c0b.view(np.uint32))
    assert np.array_equal(c0.view(np.uint32), c1.view(np.uint32))
    assert np.all(c0[:, n:] == sentinel)
    check_rows(m, n, k, a, lda, b, ldb, c0, ldc, list(range(m)) if m * n <= 1 << 20 else sample_rows(m, 8))
    assert tk_b200.device_status() == 0


def test_small_m_misaligned_operands():
    """Odd leading dimensions and misaligned bases (copied into dense buffers first) on the
    operand-swapped kernel."""
    m, n, k = 32, 1024, 512
    a, b = oracle.gen_gemm_normal(12, 0.02, m, n, k, k + 3, n + 5)
    c = run_gemm(m, n, k, a, k + 3, b, n + 5, n + 1)
    check_rows(m, n, k, a, k + 3, b, n + 5, c, n + 1, list(range(m)))


def test_small_m_kernel_and_row_tiles_agree():
    """The decode shape 16 x 4096 x 4096 on both small-M paths (the operand-swapped kernel,
    the default, and 128-row tiles): each within the error bound of the FP64 oracle."""
    m, n, k = 16, 4096, 4096
    a, b = oracle.gen_gemm_normal(3, 0.02, m, n, k, k, n)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    prev = tk_b200.lib().tk_gemm_set_small_m(1)
    try:
        for mode in (1, 0):
            tk_b200.lib().tk_gemm_set_small_m(mode)
            c = run_gemm(m, n, k, a, k, b, n, n)
            assert oracle.gemm_check(k, c, r, s, n, n)[0] == 0, mode
    finally:
        tk_b200.lib().tk_gemm_set_small_m(prev)
    assert tk_b200.device_status() == 0
