"""The restated CPU oracle against the golden fixtures made by the reference's own
host code (tests/golden/make_golden.py). CPU only; no reference tree needed."""

import hashlib
import math
import os

import numpy as np
import pytest

import oracle
from oracle import fixtures as fx

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def same(store, key, arr):
    """Bit-exact agreement with a stored array, whole or via digest + sample."""
    arr = np.ascontiguousarray(arr)
    assert tuple(store[key + "__shape"]) == arr.shape, key
    assert hashlib.sha256(arr.tobytes()).hexdigest() == str(store[key + "__sha"]), key


@pytest.mark.parametrize("case", fx.DIFFERENTIAL_EXACT_CASES + fx.DIFFERENTIAL_MODEL_CASES,
                         ids=lambda c: c[0])
def test_gemm_differential_fixture_and_reference(case):
    """Inputs (gemm_differential.cu:263-308) and R, S, bound (:380-401) bit-exact."""
    g = load("gemm_differential")
    name, m, n, k, lda, ldb, ldc, pattern = case
    a, b = fx.differential_inputs(m, n, k, lda, ldb, pattern)
    same(g, name + "/a", a)
    same(g, name + "/b", b)
    r, s = oracle.gemm_ref(m, n, k, a, lda, b, ldb)
    same(g, name + "/value", r)
    same(g, name + "/sum_abs", s)
    is_model = pattern in fx.MODEL_PATTERNS
    if is_model:
        bound = np.vectorize(lambda x: oracle.error_bound(k, x))(s)
    else:
        bound = np.zeros_like(s)
    same(g, name + "/bound", bound)


@pytest.mark.parametrize("case", fx.CORRECTNESS_CASES, ids=lambda c: c[0])
def test_gemm_correctness_fixture_and_reference(case):
    """Inputs (gemm_correctness.cu:52-89, std::mt19937) and the float reference (:91-116)."""
    name, m, n, k, lda, ldb, ldc, pattern, seed, exact = case
    if m > 1 << 20:
        a, b = fx.correctness_inputs(64, n, k, lda, ldb, pattern, seed)
        # Identity right operand: C equals A's first n columns (:96-103).
        r, _ = oracle.gemm_ref(64, n, k, a, lda, b, ldb)
        assert np.array_equal(r, oracle.f16_bits_to_f32(a[:, :n]).astype(np.float64))
        return
    g = load("gemm_correctness")
    a, b = fx.correctness_inputs(m, n, k, lda, ldb, pattern, seed)
    same(g, name + "/a", a)
    same(g, name + "/b", b)
    r, _ = oracle.gemm_ref(m, n, k, a, lda, b, ldb)
    out = np.full((m, ldc), fx.CORR_SENTINEL, dtype=np.float32)
    out[:, :n] = r.astype(np.float32)
    same(g, name + "/out", out)


def test_error_bound_table():
    """numerical_bounds.hpp:9-33 reproduced for valid and invalid metadata."""
    g = load("bounds")
    for i, k in enumerate(g["k"]):
        for j, s in enumerate(g["s"]):
            want = g["error_bound"][i, j]
            got = oracle.error_bound(int(k), float(s))
            assert (math.isnan(want) and math.isnan(got)) or (got == want and
                                                             math.copysign(1, got) == math.copysign(1, want))
    for args, want in zip(g["within_args"], g["within"]):
        assert oracle.lib().tko_within_bound(*map(float, args)) == int(want)


def test_error_bound_self_checks():
    """The reference's own self-test assertions (tests/numerical_bounds.cpp:33-87)."""
    eb = oracle.error_bound
    assert eb(16, 1.0) >= 1.0 / 262143.0
    assert 1.0 <= eb(16, 262143.0) <= 1.0 + 4 * 2.0 ** -52
    assert eb(1024, 1.0) > 0 and math.isfinite(eb(1024, 1.0))
    assert eb(16, 0.0) == 0.0 and not math.copysign(1, eb(16, -0.0)) < 0
    assert all(math.isnan(eb(k, 1.0)) for k in (0, 17, 1040))
    assert math.isfinite(eb(1024, np.finfo(np.float64).max))
    # Extended model: same values inside the reference domain, finite beyond it.
    for k in (16, 256, 1024):
        assert oracle.error_bound_extended(k, 3.0) == eb(k, 3.0)
    assert math.isfinite(oracle.error_bound_extended(8192, 3.0))
    assert math.isfinite(oracle.error_bound_extended(14336, 3.0))


def test_attention_fixtures_and_reference():
    """attention_correctness.cu fills (:40-83) and FP64 reference (:97-140) bit-exact."""
    g = load("attention")
    for which in range(5):
        q, k, v = fx.attention_inputs(which)
        q, k, v = q.reshape(-1), k.reshape(-1), v.reshape(-1)
        assert np.array_equal(q, g[f"fill{which}/q"])
        assert np.array_equal(k, g[f"fill{which}/k"])
        assert np.array_equal(v, g[f"fill{which}/v"])
        for causal in (0, 1):
            out, prob = oracle.attention_ref(q, k, v, 16, 16, 0.25, causal, want_prob=True)
            assert np.array_equal(prob.reshape(-1), g[f"fill{which}/causal{causal}/prob"])
            assert np.array_equal(oracle.f32_to_f16_bits(prob.astype(np.float32)).reshape(-1).dtype,
                                  np.dtype(np.uint16))
            rounded = np.array([oracle.lib().tko_f64_to_f16(float(x)) for x in prob.reshape(-1)],
                               dtype=np.uint16)
            assert np.array_equal(rounded, g[f"fill{which}/causal{causal}/rounded"])
            assert np.array_equal(out.reshape(-1), g[f"fill{which}/causal{causal}/out"])


def test_attention_bound_matches_reference_constant():
    """(512*2^-23 + 2^-11 + gamma(32)) * sum|V| for s = 16 (attention_correctness.cu:19-21)."""
    _, _, v = fx.attention_inputs(fx.ATT_UNIFORM)
    got = oracle.attention_bound(v, 16, 16)
    eps = 2.0 ** -23
    factor = 512 * eps + 2.0 ** -11 + (32 * eps) / (1 - 32 * eps)
    want = factor * np.abs(oracle.f16_bits_to_f32(v).astype(np.float64)).sum(axis=0)
    assert np.array_equal(got, want)


def test_row_tree_against_reference():
    """canonical_row_tree (row_reduce_reference.cuh:16-24), signed-zero ties included."""
    g = load("row_reduce")
    tiles = g["tiles"]
    sums = oracle.tile_row_reduce(tiles, "sum")
    maxs = oracle.tile_row_reduce(tiles, "max")
    assert np.array_equal(sums.view(np.uint32), g["row_sum"].view(np.uint32))
    assert np.array_equal(maxs.view(np.uint32), g["row_max"].view(np.uint32))
    # The random tiles really do round inside the tree (row_reduce.cu:449-458).
    assert g["census"][2:64].sum() > 0
    # Fixture value generators (row_reduce.cu:148-176).
    r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    assert np.array_equal(fx.row_exact_value(r, c, 1), g["exact_value_seed1"])
    assert np.array_equal(fx.row_rounded_value(r, c, 17), g["rounded_value_seed17"])


def test_row_sweep_generator_seed():
    """The row-op sweep input N(0, 4) from std::mt19937(1) is what the fixtures hold."""
    g = load("row_reduce")
    assert np.array_equal(oracle.gen_normal_f32(1, 2.0, 62 * 256).reshape(62, 16, 16), g["tiles"][2:64])


def test_softmax_logit_fixtures():
    g = load("softmax")
    for kind in range(4):
        assert np.array_equal(fx.softmax_logits(8, kind), g[f"kind{kind}"])
    for extreme in (0, 1):
        assert np.array_equal(fx.causal_logits(bool(extreme)), g[f"causal{extreme}"])


def test_softmax_reference_properties():
    """FP64 softmax (tile_softmax.cu:143-160): rows sum to 1, causal zeros exact."""
    for kind in range(4):
        logits = fx.softmax_logits(8, kind)
        want = oracle.tile_row_softmax_f64(logits, False)
        assert np.allclose(want.sum(axis=-1), 1.0, atol=1e-12)
        fails, err = oracle.tile_row_softmax_check(logits, want.astype(np.float32), False)
        assert fails == 0 and err <= oracle.SOFTMAX_BOUND
    for extreme in (False, True):
        logits = fx.causal_logits(extreme)[None]
        want = oracle.tile_row_softmax_f64(logits, True)
        r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
        assert np.all(want[0][c > r] == 0.0)
        fails, _ = oracle.tile_row_softmax_check(logits, want.astype(np.float32), True)
        assert fails == 0


def test_softmax_check_detects_planted_error():
    """The checker itself rejects an output nudged past the bound (planted on the CPU)."""
    logits = fx.softmax_logits(2, 0)
    good = oracle.tile_row_softmax_f64(logits, False).astype(np.float32)
    bad = good.copy()
    bad[1, 3, 7] += np.float32(1e-3)
    assert oracle.tile_row_softmax_check(logits, bad, False)[0] > 0
    causal = oracle.tile_row_softmax_f64(logits, True).astype(np.float32)
    causal[0, 2, 9] = np.float32(1e-30)  # a masked entry that is not exactly zero
    assert oracle.tile_row_softmax_check(logits, causal, True)[0] > 0


def test_row_softmax_check_agrees_with_tile_softmax_and_detects_errors():
    """The full-row checker on 16-column rows is the tile checker; planted errors
    (one element off, a row that no longer sums to 1) are rejected."""
    logits = fx.softmax_logits(3, 0)
    want = oracle.tile_row_softmax_f64(logits, False).astype(np.float32)
    assert oracle.row_softmax_check(logits.reshape(-1, 16), want.reshape(-1, 16))[0] == 0
    x = oracle.gen_normal_f32(8, 4.0, 6 * 1000).reshape(6, 1000)
    e = np.exp(x.astype(np.float64) - x.max(axis=1, keepdims=True))
    good = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
    assert oracle.row_softmax_check(x, good)[0] == 0
    bad = good.copy()
    bad[4, 17] += np.float32(2e-4)
    assert oracle.row_softmax_check(x, bad)[0] > 0
    scaled = good * np.float32(1.0 + 2e-4)  # every element within bound, the row sum not
    fails, _ = oracle.row_softmax_check(x, scaled)
    assert fails > 0


def test_pairwise_reduce_matches_tree():
    x = oracle.gen_normal_f32(5, 2.0, 16)
    assert oracle.pairwise_reduce(x, "sum") == oracle.lib().tko_row_tree16(x, 0)
    assert oracle.pairwise_reduce(x, "max") == oracle.lib().tko_row_tree16(x, 1)
    # 48 columns: three canonical groups, then (g0 + g1) + g2.
    y = oracle.gen_normal_f32(6, 2.0, 48)
    groups = [oracle.lib().tko_row_tree16(np.ascontiguousarray(y[16 * i:16 * i + 16]), 0) for i in range(3)]
    assert oracle.pairwise_reduce(y, "sum") == np.float32(np.float32(groups[0] + groups[1]) + groups[2])


def test_gemm_check_detects_planted_error():
    m, n, k = 32, 48, 64
    a, b = oracle.gen_gemm_uniform(2, m, n, k, k, n)
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    c = r.astype(np.float32)
    assert oracle.gemm_check(k, c, r, s, n, n)[0] == 0
    c[5, 7] += np.float32(1e-2)
    assert oracle.gemm_check(k, c, r, s, n, n)[0] == 1
