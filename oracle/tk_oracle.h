/*
 * tk_oracle.h — CPU oracle for the ThunderKittens-SM7x hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: the parity tests,
 * the smoke check and the CPU-baseline leg of the benchmark call it to produce
 * the expected results. No product code path links, loads or calls it; the
 * CUDA library under thunderkittens-sm7x_b200/ fails loudly instead of falling
 * back to anything here.
 *
 * Every function restates one host reference of ThunderKittens-SM7x (paths are
 * relative to that project's root) in plain single-threaded C++:
 *
 *   binary16 conversions   CUDA cuda_fp16.h host __float2half / __double2half /
 *                          __half2float (round-to-nearest-even), used by every
 *                          reference test; restated from IEEE 754-2008 §4.3.1.
 *   seeded generators      tests/gemm_correctness.cu:59-71 (std::mt19937 +
 *                          std::uniform_real_distribution<float>, A then B);
 *                          std::normal_distribution<float> for the other
 *                          seeded workloads.
 *   FP64 GEMM R and S      tests/gemm_differential.cu:380-401
 *   error_bound/within     tests/numerical_bounds.hpp:9-33
 *   canonical row tree     tests/row_reduce_reference.cuh:16-24 with
 *                          include/tk_sm7x/row_reduce_ops.cuh:5-15
 *   FP64 row softmax       tests/tile_softmax.cu:143-173,
 *                          tests/tile_causal_softmax.cu:74-109
 *   FP64 attention         tests/attention_correctness.cu:97-140, bound at
 *                          :19-21 and :172-177
 *
 * Parity is pinned by tests/golden/ fixtures produced by the reference's own
 * host code compiled from its sources (oracle/ref_shims, oracle/Makefile).
 */
#ifndef TK_ORACLE_H
#define TK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- binary16 ---------------------------------------------------------- */
uint16_t tko_f32_to_f16(float x);
uint16_t tko_f64_to_f16(double x);
float tko_f16_to_f32(uint16_t h);
void tko_f32_to_f16_array(const float* src, uint16_t* dst, size_t n);
void tko_f16_to_f32_array(const uint16_t* src, float* dst, size_t n);

/* ---- seeded generators --------------------------------------------------- */
/* A (m x k, leading dimension lda) then B (k x n, ldb) from one std::mt19937
 * seeded with `seed`, values uniform in [lo, hi) as float rounded to binary16.
 * Padding columns are not touched. */
void tko_gen_gemm_uniform(uint32_t seed, float lo, float hi, int m, int n, int k,
                          uint16_t* a, int lda, uint16_t* b, int ldb);
/* Same order, values std::normal_distribution<float>(0, sigma). */
void tko_gen_gemm_normal(uint32_t seed, float sigma, int m, int n, int k,
                         uint16_t* a, int lda, uint16_t* b, int ldb);
/* `count` FP32 values N(0, sigma^2) from std::mt19937(seed). */
void tko_gen_normal_f32(uint32_t seed, float sigma, float* out, size_t count);
/* Q, then K, then V (each `count` binary16 values, N(0, sigma^2)) from one
 * std::mt19937(seed). */
void tko_gen_qkv_normal(uint32_t seed, float sigma, size_t count, uint16_t* q,
                        uint16_t* k, uint16_t* v);

/* ---- GEMM ------------------------------------------------------------------ */
/* Per output cell: r = sum_k a*b and s = sum_k |a*b| in binary64, summed in
 * index order (tests/gemm_differential.cu:380-401). r or s may be NULL.
 * Output leading dimension ldr. */
void tko_gemm_ref_f64(int m, int n, int k, const uint16_t* a, int lda,
                      const uint16_t* b, int ldb, double* r, double* s, int ldr);
/* tests/numerical_bounds.hpp:9-28: NaN unless 16 <= k <= 1024, k % 16 == 0. */
double tko_error_bound(int k, double sum_abs);
/* Same formula with no upper cap on k (extrapolated model for k > 1024). */
double tko_error_bound_extended(int k, double sum_abs);
/* tests/numerical_bounds.hpp:30-33 */
int tko_within_bound(double actual, double reference, double bound);
/* Checks a GPU output c (m x n, ldc) against r/s: counts cells outside the
 * (extended) bound, and cells in ldc padding that differ from `sentinel_bits`.
 * Returns the count of failures; max_ratio gets max |c-r|/E. */
size_t tko_gemm_check(int m, int n, int k, const float* c, int ldc,
                      const double* r, const double* s, int ldr,
                      uint32_t sentinel_bits, int check_padding,
                      double* max_abs, double* max_ratio);

/* ---- tile row reductions --------------------------------------------------- */
/* Balanced column-order tree of one 16-float row. op: 0 = sum, 1 = max. */
float tko_row_tree16(const float* row, int op);
/* n_tiles 16x16 row-major FP32 tiles -> 16 results per tile. */
void tko_tile_row_reduce(const float* tiles, size_t n_tiles, float* out, int op);
/* Level-by-level pairwise reduction over n values (stride apart): pairs
 * (2i, 2i+1) combine low-then-high; an odd last element is carried up. For
 * n = 16 it equals the canonical tree; for n = 16*g it equals the canonical
 * tree per 16-column group followed by the same pairwise rule over groups. */
float tko_pairwise_reduce(const float* x, size_t n, size_t stride, int op);
/* Per-row pairwise max and sum of an m x n FP32 matrix (ldc). */
void tko_matrix_row_stats(const float* c, int m, int n, int ldc, float* row_max,
                          float* row_sum);

/* ---- tile row softmax ------------------------------------------------------ */
/* FP64 reference of exp(x - max) / sum per row (tests/tile_softmax.cu:143-160);
 * causal: row i uses columns 0..i and the rest are exactly 0
 * (tests/tile_causal_softmax.cu:74-90). */
void tko_tile_row_softmax_f64(const float* tiles, size_t n_tiles, double* out,
                              int causal);
/* Checks got (n_tiles x 256 FP32) against the FP64 reference: |got-want| <=
 * bound, 0 <= got <= 1, |row sum - 1| <= bound, causal zeros exact. Returns the
 * number of failing values (+ failing rows); max_err gets max |got - want|. */
size_t tko_tile_row_softmax_check(const float* tiles, const float* got,
                                  size_t n_tiles, int causal, double bound,
                                  double* max_err);

/* Softmax over full rows of length n (row pitch ldx / ldg); same checks, FP64. */
size_t tko_row_softmax_check(const float* x, size_t m, size_t n, size_t ldx, const float* got,
                             size_t ldg, double bound, double* max_err);

/* ---- attention ------------------------------------------------------------- */
/* One (batch, head) slice: q, k, v are s x d row-major binary16. For query rows
 * [row_begin, row_end): FP64 scores * scale, max over allowed keys, exp,
 * normalise, round the probability to binary16 (RNE, from binary64), FP64
 * P.V -> out ((row_end-row_begin) x d). causal: key t allowed iff t <= row.
 * tests/attention_correctness.cu:97-140 generalised to s x d and any scale.
 * prob (optional, rows x s) receives the unrounded FP64 probabilities. */
void tko_attention_ref_f64(const uint16_t* q, const uint16_t* k,
                           const uint16_t* v, int s, int d, double scale,
                           int causal, int row_begin, int row_end, double* out,
                           double* prob);
/* Per output column c: (512*2^-23 + 2^-11 + gamma(2s)) * sum_t |v[t, c]|
 * (tests/attention_correctness.cu:19-21, 172-177 with gamma(32) -> gamma(2s)). */
void tko_attention_bound(const uint16_t* v, int s, int d, double* bound_per_col);

#ifdef __cplusplus
}
#endif

#endif /* TK_ORACLE_H */
