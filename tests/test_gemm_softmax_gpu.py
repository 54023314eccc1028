"""Fused GEMM -> full-row softmax on the GPU through the C ABI.

C is checked against the FP64 GEMM oracle with the GEMM bound; P against the FP64
softmax of each row of the C the GPU returned, with the reference's softmax bound
512 * 2^-23 per element and on each row sum (tests/tile_softmax.cu:20,160-173),
generalising examples/gemm_row_softmax.cu:25-48 from one 16x16 tile to rows of
any length."""

import numpy as np
import pytest
import torch

import oracle
import tk_b200
from cuda_util import dev, host

pytestmark = pytest.mark.gpu


def run(m, n, k, sigma, seed, cta_group=0, in_place=False):
    a, b = oracle.gen_gemm_normal(seed, sigma, m, n, k, k, n)
    da, db = dev(a), dev(b)
    prev = tk_b200.set_gemm_cta_group(cta_group)
    try:
        c, p = tk_b200.gemm_rowsoftmax(da, db, in_place=in_place)
    finally:
        tk_b200.set_gemm_cta_group(prev)
    return a, b, host(c), host(p)


@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("shape", [(16, 16, 16), (128, 256, 64), (256, 384, 512), (400, 1008, 256),
                                   (272, 4096, 128), (128, 16384, 64)],
                         ids=lambda s: "x".join(map(str, s)))
def test_rowsoftmax_matches_oracle(shape, cta_group):
    m, n, k = shape
    sigma = (3.0 / np.sqrt(k)) ** 0.5  # C has standard deviation about 3
    a, b, c, p = run(m, n, k, sigma, seed=m + n + k, cta_group=cta_group)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    assert oracle.gemm_check(k, c, r, s, n, n)[0] == 0
    fails, err = oracle.row_softmax_check(c, p)
    assert fails == 0, err


def test_rowsoftmax_wide_logits():
    """Logits with a spread of hundreds: most probabilities underflow to 0, the row
    max carries almost all the mass."""
    m, n, k = 256, 2048, 256
    a, b, c, p = run(m, n, k, sigma=1.5, seed=9)
    assert np.ptp(c) > 200
    fails, err = oracle.row_softmax_check(c, p)
    assert fails == 0, err


def test_rowsoftmax_in_place_equals_separate_output():
    m, n, k = 384, 1280, 192
    sigma = (3.0 / np.sqrt(k)) ** 0.5
    _, _, c, p = run(m, n, k, sigma, seed=3)
    _, _, c2, p2 = run(m, n, k, sigma, seed=3, in_place=True)
    assert np.array_equal(p2.view(np.uint32), p.view(np.uint32))
    assert oracle.row_softmax_check(c, p2)[0] == 0


def test_rowsoftmax_strided_outputs_keep_padding():
    """ldc and ldp wider than n: the padding columns of C and P are untouched."""
    m, n, k, ldc, ldp = 144, 528, 96, 600, 532
    sigma = (3.0 / np.sqrt(k)) ** 0.5
    a, b = oracle.gen_gemm_normal(11, sigma, m, n, k, k, n)
    da, db = dev(a), dev(b)
    c = torch.full((m, ldc), -7.0, device="cuda")
    p = torch.full((m, ldp), -9.0, device="cuda")
    assert tk_b200.gemm_rowsoftmax_raw(m, n, k, da, k, db, n, c, ldc, p, ldp) == 0
    ch, ph = host(c), host(p)
    assert np.all(ch[:, n:] == -7.0) and np.all(ph[:, n:] == -9.0)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    assert oracle.gemm_check(k, ch[:, :n], r, s, n, n)[0] == 0
    assert oracle.row_softmax_check(ch[:, :n], ph[:, :n])[0] == 0


def test_rowsoftmax_8192x8192x8192_sampled_rows():
    m = n = k = 8192
    sigma = (3.0 / np.sqrt(k)) ** 0.5
    a, b = oracle.gen_gemm_normal(4, sigma, m, n, k, k, n)
    da, db = dev(a), dev(b)
    c, p = tk_b200.gemm_rowsoftmax(da, db)
    c, p = host(c), host(p)
    rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(0).integers(0, m, 24)]))
    fails, err = oracle.row_softmax_check(c[rows], p[rows])
    assert fails == 0, err
    sums = p.astype(np.float64).sum(axis=1)
    assert np.all(np.abs(sums - 1.0) <= oracle.SOFTMAX_BOUND)
