"""Restated fixture generators of the ThunderKittens-SM7x test suite (test infrastructure).

These produce the same input bits as the reference tests' host fill functions; the
golden files in tests/golden/ (made from the reference's own compiled fill code)
pin them. File:line citations are relative to the reference project root.
"""

from __future__ import annotations

import numpy as np

from . import f32_to_f16_bits, gen_gemm_uniform

# tests/gemm_differential.cu:32-43
IDENTITY, SIGNED_SEED_A, SIGNED_SEED_B, CANCELLATION = 0, 1, 2, 3
ROUNDED_POSITIVE, ROUNDED_SIGNED, ROUNDED_MIXED, ROUNDED_MIXED_ZEROS = 4, 5, 6, 7
ROUNDED_CANCELLATION, ROUNDED_ZERO = 8, 9
MODEL_PATTERNS = {ROUNDED_POSITIVE, ROUNDED_SIGNED, ROUNDED_MIXED, ROUNDED_MIXED_ZEROS,
                  ROUNDED_CANCELLATION, ROUNDED_ZERO}

# tests/gemm_differential.cu:691-698 (exact-domain roster) and :642-653 (model roster):
# (name, m, n, k, lda, ldb, ldc, pattern)
DIFFERENTIAL_EXACT_CASES = [
    ("identity", 16, 16, 16, 24, 24, 20, IDENTITY),
    ("signed-multi-cta", 32, 48, 32, 40, 56, 52, SIGNED_SEED_A),
    ("long-k", 16, 32, 1024, 1032, 40, 36, SIGNED_SEED_B),
    ("cancellation", 16, 16, 64, 72, 24, 20, CANCELLATION),
    ("production-small", 256, 384, 32, 40, 392, 388, SIGNED_SEED_A),
    ("production-large", 1024, 1024, 32, 40, 1032, 1028, SIGNED_SEED_B),
]
DIFFERENTIAL_MODEL_CASES = [
    ("rounded-positive-short", 16, 16, 16, 24, 24, 20, ROUNDED_POSITIVE),
    ("rounded-positive-long", 16, 16, 1024, 1032, 24, 20, ROUNDED_POSITIVE),
    ("rounded-signed", 32, 48, 256, 264, 56, 52, ROUNDED_SIGNED),
    ("rounded-mixed", 32, 48, 256, 264, 56, 52, ROUNDED_MIXED),
    ("rounded-mixed-long", 32, 48, 1024, 1032, 56, 52, ROUNDED_MIXED),
    ("rounded-mixed-zeros", 32, 48, 256, 264, 56, 52, ROUNDED_MIXED_ZEROS),
    ("rounded-cancellation", 16, 32, 1024, 1032, 40, 36, ROUNDED_CANCELLATION),
    ("rounded-zero", 16, 16, 32, 40, 24, 20, ROUNDED_ZERO),
    ("rounded-production-small", 256, 384, 64, 72, 392, 388, ROUNDED_MIXED),
    ("rounded-production-large", 1024, 1024, 32, 40, 1032, 1028, ROUNDED_MIXED),
]

# tests/gemm_correctness.cu:18-22 patterns and :434-449 roster:
# (name, m, n, k, lda, ldb, ldc, pattern, seed, exact)
CORR_IDENTITY_RIGHT, CORR_FINGERPRINT, CORR_RANDOM = 0, 1, 2
CORRECTNESS_CASES = [
    ("identity-16x16x16", 16, 16, 16, 16, 16, 16, CORR_IDENTITY_RIGHT, 0, True),
    ("identity-8388608x16x16-grid-y-boundary", 8388608, 16, 16, 16, 16, 16,
     CORR_IDENTITY_RIGHT, 0, True),
    ("fingerprint-16x16x32", 16, 16, 32, 32, 16, 16, CORR_FINGERPRINT, 0, True),
    ("random-32x48x32-strided", 32, 48, 32, 37, 53, 59, CORR_RANDOM, 0x75C0FFEE, False),
    ("random-32x32x48", 32, 32, 48, 48, 32, 32, CORR_RANDOM, 0x70C0FFEE, False),
    ("random-256x384x32-strided-small-tile", 256, 384, 32, 41, 397, 401, CORR_RANDOM,
     0x5EED1234, False),
    ("random-1024x1024x32-strided-large-tile", 1024, 1024, 32, 37, 1039, 1051, CORR_RANDOM,
     0x1A2B3C4D, False),
]
CORR_SENTINEL = np.float32(-123456.0)  # tests/gemm_correctness.cu:16


def _half(values) -> np.ndarray:
    return f32_to_f16_bits(np.asarray(values, dtype=np.float32))


def fingerprint(row, col, seed) -> np.ndarray:
    """tests/gemm_differential.cu:205-213 (uint32 wrap-around hash)."""
    row = np.asarray(row, dtype=np.uint64)
    col = np.asarray(col, dtype=np.uint64)
    mask = np.uint64(0xFFFFFFFF)
    v = ((row * np.uint64(0x9E3779B9)) & mask) ^ ((col * np.uint64(0x85EBCA6B)) & mask) ^ np.uint64(seed)
    v ^= v >> np.uint64(16)
    v = (v * np.uint64(0x7FEB352D)) & mask
    v ^= v >> np.uint64(15)
    v = (v * np.uint64(0x846CA68B)) & mask
    return (v ^ (v >> np.uint64(16))) & mask


def rounded_value(h, pattern, negate) -> np.ndarray:
    """tests/gemm_differential.cu:215-224."""
    h = np.asarray(h, dtype=np.uint64)
    if pattern in (ROUNDED_MIXED, ROUNDED_MIXED_ZEROS):
        exponent = ((h >> np.uint64(10)) % np.uint64(7)).astype(np.int64) - 3
    else:
        exponent = np.zeros(h.shape, dtype=np.int64)
    value = np.ldexp(np.float32(1.0) + (h & np.uint64(1023)).astype(np.float32) / np.float32(1024.0),
                     exponent).astype(np.float32)
    neg = np.broadcast_to(np.asarray(negate, dtype=bool), h.shape).copy()
    if pattern in (ROUNDED_SIGNED, ROUNDED_MIXED, ROUNDED_MIXED_ZEROS):
        neg |= (h >> np.uint64(31)) != 0
    value = np.where(neg, -value, value)
    return _half(value)


def value_from_q(q) -> np.ndarray:
    return _half(np.asarray(q, dtype=np.float32) / np.float32(8.0))


def signed_q(row, col, seed):
    return (row * 3 + col * 5 + seed) % 17 - 8


def differential_inputs(m, n, k, lda, ldb, pattern):
    """tests/gemm_differential.cu:263-308: A (m x lda), B (k x ldb) as binary16 bits.

    Padding holds q = 7 (7/8), a nonzero value so reading it corrupts results."""
    a = np.full((m, lda), value_from_q(7), dtype=np.uint16)
    b = np.full((k, ldb), value_from_q(7), dtype=np.uint16)
    rows_a, cols_a = np.meshgrid(np.arange(m), np.arange(k), indexing="ij")
    rows_b, cols_b = np.meshgrid(np.arange(k), np.arange(n), indexing="ij")
    if pattern in MODEL_PATTERNS:
        if pattern == ROUNDED_CANCELLATION:
            coord = cols_a % (k // 2)
            negate = cols_a >= k // 2
        else:
            coord = cols_a
            negate = np.zeros_like(cols_a, dtype=bool)
        va = rounded_value(fingerprint(rows_a, coord, 17), pattern, negate)
        if pattern == ROUNDED_ZERO:
            va[...] = _half(0.0)
        if pattern == ROUNDED_MIXED_ZEROS:
            va[cols_a % 4 == 0] = _half(0.0)
        a[:, :k] = va
        coord_b = rows_b % (k // 2) if pattern == ROUNDED_CANCELLATION else rows_b
        b[:, :n] = rounded_value(fingerprint(coord_b, cols_b, 83), pattern, False)
        return a, b
    if pattern == CANCELLATION:
        qa = np.where(cols_a % 2 == 0, 8, -8)
    else:
        qa = signed_q(rows_a, cols_a, 1 if pattern == SIGNED_SEED_A else 9)
    a[:, :k] = value_from_q(qa)
    qb = signed_q(rows_b, cols_b, 11 if pattern == SIGNED_SEED_A else 3)
    if pattern == IDENTITY:
        qb = np.where(rows_b == cols_b, 8, 0)
    if pattern == CANCELLATION:
        qb = np.full_like(qb, 8)
    b[:, :n] = value_from_q(qb)
    return a, b


def correctness_inputs(m, n, k, lda, ldb, pattern, seed):
    """tests/gemm_correctness.cu:52-89 (padding stays zero)."""
    if pattern == CORR_RANDOM:
        return gen_gemm_uniform(seed, m, n, k, lda, ldb)
    a = np.zeros((m, lda), dtype=np.uint16)
    b = np.zeros((k, ldb), dtype=np.uint16)
    rows_a, cols_a = np.meshgrid(np.arange(m), np.arange(k), indexing="ij")
    a[:, :k] = _half((rows_a * 3 + cols_a * 5) % 7 - 3)
    rows_b, cols_b = np.meshgrid(np.arange(k), np.arange(n), indexing="ij")
    if pattern == CORR_IDENTITY_RIGHT:
        b[:, :n] = _half(np.where(rows_b == cols_b, 1.0, 0.0))
    else:
        b[:, :n] = _half((rows_b * 2 + cols_b * 3) % 5 - 2)
    return a, b


# ---- attention (tests/attention_correctness.cu:40-83) -------------------------------
ATT_UNIFORM, ATT_SHIFTED_IDENTITY, ATT_SHIFTED_ASYM, ATT_LARGE, ATT_ALIAS = 0, 1, 2, 3, 4


def attention_inputs(which):
    """Returns q, k, v (16x16 binary16 bits); ATT_ALIAS returns q three times."""
    r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    asym = ((3 * r + 5 * c) % 13 - 6) / 8.0
    if which == ATT_UNIFORM:
        q = np.zeros((16, 16))
        k = ((7 * r + c) % 11 - 5) / 8.0
        v = asym
    elif which in (ATT_SHIFTED_IDENTITY, ATT_SHIFTED_ASYM):
        onehot = c == (r + 1) % 16
        q = np.where(onehot, 4.0, 0.0)
        k = np.where(onehot, 2.0, 0.0)
        v = np.where(r == c, 1.0, 0.0) if which == ATT_SHIFTED_IDENTITY else asym
    elif which == ATT_LARGE:
        q = np.where(r == c, 64.0, 0.0)
        k = np.where(r == c, 64.0, 0.0)
        v = np.where(r == c, 1.0, 0.0)
    else:
        q = asym
        return _half(q), _half(q), _half(q)
    return _half(q), _half(k), _half(v)


# (name, fill, causal, exact_uniform, midpoint_favored, exact_large, identity_v):
# tests/attention_correctness.cu:263-324
ATTENTION_CASES = [
    ("uniform scores", ATT_UNIFORM, False, True, False, False, False),
    ("shifted K, identity V", ATT_SHIFTED_IDENTITY, False, False, True, False, False),
    ("shifted K, asymmetric V", ATT_SHIFTED_ASYM, False, False, False, False, False),
    ("large finite scores", ATT_LARGE, False, False, False, True, False),
    ("aliased Q/K/V", ATT_ALIAS, False, False, False, False, False),
    ("causal uniform scores", ATT_UNIFORM, True, False, False, False, False),
    ("causal shifted K, identity V", ATT_SHIFTED_IDENTITY, True, False, False, False, True),
    ("causal shifted K, asymmetric V", ATT_SHIFTED_ASYM, True, False, False, False, False),
    ("causal large finite scores", ATT_LARGE, True, False, False, True, True),
    ("causal aliased Q/K/V", ATT_ALIAS, True, False, False, False, False),
]


def attention_exact_mask(exact_uniform, midpoint_favored, exact_large, causal, identity_v):
    """Cells that must equal the FP64 reference exactly (tests/attention_correctness.cu:180-182)."""
    r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    mask = np.zeros((16, 16), dtype=bool)
    if exact_uniform or exact_large:
        mask[...] = True
    if midpoint_favored:
        mask |= r == c
    if causal:
        mask |= r == 0
        if identity_v:
            mask |= c > r
    return mask


# ---- row reductions (tests/row_reduce.cu:148-176, tests/tile_reduce.cu:55-91) ------

def row_exact_value(row, col, seed):
    return _half(((row * 3 + col * 5 + seed) % 17 - 8) / 8.0)


def row_rounded_value(row, col, seed):
    return rounded_value(fingerprint(row, col, seed), ROUNDED_MIXED, False)


# ---- softmax logits (tests/tile_softmax.cu:97-108, tests/tile_causal_softmax.cu:270-273)

def softmax_logits(groups, kind) -> np.ndarray:
    """(groups, 16, 16) FP32 logits of the reference's four softmax fixture kinds."""
    g, r, c = np.meshgrid(np.arange(groups), np.arange(16), np.arange(16), indexing="ij")
    if kind == 1:
        return np.zeros((groups, 16, 16), dtype=np.float32)
    if kind == 2:
        base = np.where(r % 2 == 0, np.float32(1000.0), np.float32(-1000.0)).astype(np.float32)
        return (base + ((c + r + g).astype(np.float32) / np.float32(2.0))).astype(np.float32)
    if kind == 3:
        mantissa = 1024 + (137 * r + 79 * c + 53 * g) % 1024
        exponent = (r + 2 * c + g) % 7 - 3
        return np.ldexp(mantissa.astype(np.float32), exponent - 10).astype(np.float32)
    v = (((5 * c + 3 * r + 7 * g) % 16 - 8).astype(np.float32) / np.float32(8.0)
         + r.astype(np.float32) / np.float32(2.0) + g.astype(np.float32) / np.float32(4.0))
    return v.astype(np.float32)


def causal_logits(extreme: bool) -> np.ndarray:
    r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    if extreme:
        return np.full((16, 16), -np.finfo(np.float32).max, dtype=np.float32)
    return (((3 * r + 5 * c) % 13 - 6) / 8.0).astype(np.float32)
