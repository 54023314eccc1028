// tk_oracle.cpp — CPU oracle for the ThunderKittens-SM7x hot path.
//
// TEST INFRASTRUCTURE ONLY: the checker used by tests/, __graft_entry__.smoke()
// and the CPU-baseline leg of bench.py. Nothing on the product path calls it.
// Each function names the reference file:line it restates (paths relative to
// the ThunderKittens-SM7x project root).

#include "tk_oracle.h"

#include <cfenv>
#include <cmath>
#include <cstring>
#include <limits>
#include <random>
#include <vector>

namespace {

// IEEE 754 binary16 from a binary64 value, one rounding, to nearest even.
// Both float and double inputs go through this: a float converts to double
// exactly, so the single rounding below is the float -> half rounding too.
// Semantics follow CUDA's host __float2half / __double2half (RNE, overflow to
// infinity, gradual underflow); NaN maps to the canonical 0x7fff.
uint16_t to_half(double x) {
    uint16_t sign = std::signbit(x) ? 0x8000u : 0u;
    if (std::isnan(x)) return 0x7fffu;
    double a = std::fabs(x);
    if (std::isinf(a)) return sign | 0x7c00u;
    if (a == 0.0) return sign;
    if (a < 0x1p-14) {
        // Subnormal range: units of 2^-24. Scaling by a power of two is exact.
        double q = std::nearbyint(a * 0x1p24);  // default mode: to nearest even
        return sign | static_cast<uint16_t>(q);  // q == 1024 is the smallest normal
    }
    int e2 = 0;
    std::frexp(a, &e2);          // a = f * 2^e2, f in [0.5, 1)
    int e = e2 - 1;              // a in [2^e, 2^(e+1))
    double m = std::nearbyint(std::ldexp(a, 10 - e));  // in [1024, 2048]
    if (m == 2048.0) {
        m = 1024.0;
        e += 1;
    }
    if (e > 15) return sign | 0x7c00u;
    return sign | static_cast<uint16_t>(((e + 15) << 10) | (static_cast<int>(m) - 1024));
}

double half_value(uint16_t h) {
    int exponent = (h >> 10) & 0x1f;
    int fraction = h & 0x3ff;
    double mag;
    if (exponent == 0) {
        mag = std::ldexp(static_cast<double>(fraction), -24);
    } else if (exponent == 31) {
        mag = fraction == 0 ? std::numeric_limits<double>::infinity()
                            : std::numeric_limits<double>::quiet_NaN();
    } else {
        mag = std::ldexp(static_cast<double>(1024 + fraction), exponent - 25);
    }
    return (h & 0x8000u) ? -mag : mag;
}

// include/tk_sm7x/row_reduce_ops.cuh:5-15
inline float combine(float low, float high, int op) {
    if (op == 0) return low + high;
    return low > high ? low : high;
}

double gamma_up(int k) {
    constexpr double epsilon = 0x1p-23;
    const double n = 2.0 * static_cast<double>(k);
    return std::nextafter(n * epsilon / (1.0 - n * epsilon),
                          std::numeric_limits<double>::infinity());
}

double bound_from(int k, double sum_abs) {
    if (sum_abs == 0.0) return 0.0;
    const double bound = std::nextafter(gamma_up(k) * sum_abs,
                                        std::numeric_limits<double>::infinity());
    if (!std::isfinite(bound)) return std::numeric_limits<double>::quiet_NaN();
    return bound;
}

}  // namespace

extern "C" {

uint16_t tko_f32_to_f16(float x) { return to_half(static_cast<double>(x)); }
uint16_t tko_f64_to_f16(double x) { return to_half(x); }
float tko_f16_to_f32(uint16_t h) { return static_cast<float>(half_value(h)); }

void tko_f32_to_f16_array(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = to_half(static_cast<double>(src[i]));
}

void tko_f16_to_f32_array(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = static_cast<float>(half_value(src[i]));
}

// tests/gemm_correctness.cu:59-71: one generator, A row-major then B row-major.
void tko_gen_gemm_uniform(uint32_t seed, float lo, float hi, int m, int n, int k,
                          uint16_t* a, int lda, uint16_t* b, int ldb) {
    std::mt19937 generator(seed);
    std::uniform_real_distribution<float> distribution(lo, hi);
    for (int row = 0; row < m; ++row)
        for (int col = 0; col < k; ++col)
            a[static_cast<size_t>(row) * lda + col] = to_half(distribution(generator));
    for (int row = 0; row < k; ++row)
        for (int col = 0; col < n; ++col)
            b[static_cast<size_t>(row) * ldb + col] = to_half(distribution(generator));
}

void tko_gen_gemm_normal(uint32_t seed, float sigma, int m, int n, int k,
                         uint16_t* a, int lda, uint16_t* b, int ldb) {
    std::mt19937 generator(seed);
    std::normal_distribution<float> distribution(0.0f, sigma);
    for (int row = 0; row < m; ++row)
        for (int col = 0; col < k; ++col)
            a[static_cast<size_t>(row) * lda + col] = to_half(distribution(generator));
    for (int row = 0; row < k; ++row)
        for (int col = 0; col < n; ++col)
            b[static_cast<size_t>(row) * ldb + col] = to_half(distribution(generator));
}

void tko_gen_normal_f32(uint32_t seed, float sigma, float* out, size_t count) {
    std::mt19937 generator(seed);
    std::normal_distribution<float> distribution(0.0f, sigma);
    for (size_t i = 0; i < count; ++i) out[i] = distribution(generator);
}

void tko_gen_qkv_normal(uint32_t seed, float sigma, size_t count, uint16_t* q,
                        uint16_t* k, uint16_t* v) {
    std::mt19937 generator(seed);
    std::normal_distribution<float> distribution(0.0f, sigma);
    for (size_t i = 0; i < count; ++i) q[i] = to_half(distribution(generator));
    for (size_t i = 0; i < count; ++i) k[i] = to_half(distribution(generator));
    for (size_t i = 0; i < count; ++i) v[i] = to_half(distribution(generator));
}

// tests/gemm_differential.cu:380-401: binary64 products of the binary16 inputs
// summed in k order; s is the sum of absolute products.
void tko_gemm_ref_f64(int m, int n, int k, const uint16_t* a, int lda,
                      const uint16_t* b, int ldb, double* r, double* s, int ldr) {
    std::vector<double> brow(static_cast<size_t>(k));
    std::vector<double> acol(static_cast<size_t>(k));
    // Convert B column-by-column lazily would be slow; convert B once.
    std::vector<double> bd(static_cast<size_t>(k) * n);
    for (int kk = 0; kk < k; ++kk)
        for (int col = 0; col < n; ++col)
            bd[static_cast<size_t>(kk) * n + col] = half_value(b[static_cast<size_t>(kk) * ldb + col]);
    std::vector<double> sum(n), sum_abs(n);
    for (int row = 0; row < m; ++row) {
        for (int kk = 0; kk < k; ++kk) acol[kk] = half_value(a[static_cast<size_t>(row) * lda + kk]);
        std::fill(sum.begin(), sum.end(), 0.0);
        std::fill(sum_abs.begin(), sum_abs.end(), 0.0);
        // Loop order k-outer keeps each cell's additions in k order.
        for (int kk = 0; kk < k; ++kk) {
            const double av = acol[kk];
            const double* bp = &bd[static_cast<size_t>(kk) * n];
            for (int col = 0; col < n; ++col) {
                const double product = av * bp[col];
                sum[col] += product;
                sum_abs[col] += std::fabs(product);
            }
        }
        for (int col = 0; col < n; ++col) {
            if (r) r[static_cast<size_t>(row) * ldr + col] = sum[col];
            if (s) s[static_cast<size_t>(row) * ldr + col] = sum_abs[col];
        }
    }
}

// tests/numerical_bounds.hpp:9-28
double tko_error_bound(int k, double sum_abs) {
    if (k <= 0 || k % 16 != 0 || k > 1024 || sum_abs < 0.0 || !std::isfinite(sum_abs))
        return std::numeric_limits<double>::quiet_NaN();
    return bound_from(k, sum_abs);
}

double tko_error_bound_extended(int k, double sum_abs) {
    if (k <= 0 || k % 16 != 0 || sum_abs < 0.0 || !std::isfinite(sum_abs))
        return std::numeric_limits<double>::quiet_NaN();
    if (2.0 * k * 0x1p-23 >= 1.0) return std::numeric_limits<double>::quiet_NaN();
    return bound_from(k, sum_abs);
}

// tests/numerical_bounds.hpp:30-33
int tko_within_bound(double actual, double reference, double bound) {
    return std::isfinite(actual) && std::isfinite(reference) && std::isfinite(bound) &&
           bound >= 0.0 && std::fabs(actual - reference) <= bound;
}

size_t tko_gemm_check(int m, int n, int k, const float* c, int ldc,
                      const double* r, const double* s, int ldr,
                      uint32_t sentinel_bits, int check_padding,
                      double* max_abs, double* max_ratio) {
    size_t failures = 0;
    double worst_abs = 0.0, worst_ratio = 0.0;
    for (int row = 0; row < m; ++row) {
        for (int col = 0; col < n; ++col) {
            const double got = c[static_cast<size_t>(row) * ldc + col];
            const double want = r[static_cast<size_t>(row) * ldr + col];
            const double bound = tko_error_bound_extended(k, s[static_cast<size_t>(row) * ldr + col]);
            const double err = std::fabs(got - want);
            if (std::isfinite(err) && err > worst_abs) worst_abs = err;
            const double ratio = bound == 0.0 ? (err == 0.0 ? 0.0 : INFINITY) : err / bound;
            if (!(ratio <= worst_ratio)) worst_ratio = ratio;
            if (!tko_within_bound(got, want, bound)) ++failures;
        }
        if (check_padding) {
            for (int col = n; col < ldc; ++col) {
                uint32_t bits;
                std::memcpy(&bits, &c[static_cast<size_t>(row) * ldc + col], 4);
                if (bits != sentinel_bits) ++failures;
            }
        }
    }
    if (max_abs) *max_abs = worst_abs;
    if (max_ratio) *max_ratio = worst_ratio;
    return failures;
}

// tests/row_reduce_reference.cuh:16-24 (canonical_row_tree) with the combine
// rules of include/tk_sm7x/row_reduce_ops.cuh:5-15.
float tko_row_tree16(const float* row, int op) {
    const float q0 = combine(combine(row[0], row[1], op), combine(row[2], row[3], op), op);
    const float q1 = combine(combine(row[4], row[5], op), combine(row[6], row[7], op), op);
    const float q2 = combine(combine(row[8], row[9], op), combine(row[10], row[11], op), op);
    const float q3 = combine(combine(row[12], row[13], op), combine(row[14], row[15], op), op);
    return combine(combine(q0, q1, op), combine(q2, q3, op), op);
}

void tko_tile_row_reduce(const float* tiles, size_t n_tiles, float* out, int op) {
    for (size_t t = 0; t < n_tiles; ++t)
        for (int row = 0; row < 16; ++row)
            out[t * 16 + row] = tko_row_tree16(tiles + t * 256 + row * 16, op);
}

float tko_pairwise_reduce(const float* x, size_t n, size_t stride, int op) {
    if (n == 0) return op == 0 ? 0.0f : -INFINITY;
    std::vector<float> level(n);
    for (size_t i = 0; i < n; ++i) level[i] = x[i * stride];
    size_t count = n;
    while (count > 1) {
        size_t next = 0;
        for (size_t i = 0; i + 1 < count; i += 2) level[next++] = combine(level[i], level[i + 1], op);
        if (count & 1) level[next++] = level[count - 1];
        count = next;
    }
    return level[0];
}

void tko_matrix_row_stats(const float* c, int m, int n, int ldc, float* row_max,
                          float* row_sum) {
    for (int row = 0; row < m; ++row) {
        const float* p = c + static_cast<size_t>(row) * ldc;
        if (row_max) row_max[row] = tko_pairwise_reduce(p, n, 1, 1);
        if (row_sum) row_sum[row] = tko_pairwise_reduce(p, n, 1, 0);
    }
}

// tests/tile_softmax.cu:143-160 and tests/tile_causal_softmax.cu:74-88.
void tko_tile_row_softmax_f64(const float* tiles, size_t n_tiles, double* out,
                              int causal) {
    for (size_t t = 0; t < n_tiles; ++t) {
        for (int r = 0; r < 16; ++r) {
            const float* row = tiles + t * 256 + r * 16;
            double* dst = out + t * 256 + r * 16;
            const int last = causal ? r : 15;
            double maximum = -std::numeric_limits<double>::infinity();
            for (int c = 0; c <= last; ++c) maximum = std::fmax(maximum, static_cast<double>(row[c]));
            double exponent[16], sum = 0.0;
            for (int c = 0; c <= last; ++c) {
                exponent[c] = std::exp(static_cast<double>(row[c]) - maximum);
                sum += exponent[c];
            }
            for (int c = 0; c < 16; ++c) dst[c] = c <= last ? exponent[c] / sum : 0.0;
        }
    }
}

// Checks of tests/tile_softmax.cu:160-173 and tests/tile_causal_softmax.cu:86-110.
size_t tko_tile_row_softmax_check(const float* tiles, const float* got,
                                  size_t n_tiles, int causal, double bound,
                                  double* max_err) {
    size_t failures = 0;
    double worst = 0.0;
    double want[256];
    for (size_t t = 0; t < n_tiles; ++t) {
        tko_tile_row_softmax_f64(tiles + t * 256, 1, want, causal);
        for (int r = 0; r < 16; ++r) {
            double row_sum = 0.0;
            for (int c = 0; c < 16; ++c) {
                const float g = got[t * 256 + r * 16 + c];
                const double w = want[r * 16 + c];
                const double err = std::fabs(static_cast<double>(g) - w);
                if (std::isfinite(err) && err > worst) worst = err;
                bool ok;
                if (causal && c > r) {
                    ok = (g == 0.0f);
                } else {
                    ok = std::isfinite(g) && g >= 0.0f && g <= 1.0f && err <= bound;
                }
                if (!ok) ++failures;
                row_sum += static_cast<double>(g);
            }
            if (!(std::fabs(row_sum - 1.0) <= bound)) ++failures;
        }
    }
    if (max_err) *max_err = worst;
    return failures;
}

// tests/attention_correctness.cu:97-140, generalised from one 16x16 tile with
// scale 0.25 to an s x d slice with any scale.
void tko_attention_ref_f64(const uint16_t* q, const uint16_t* k,
                           const uint16_t* v, int s, int d, double scale,
                           int causal, int row_begin, int row_end, double* out,
                           double* prob) {
    std::vector<double> kd(static_cast<size_t>(s) * d), vd(static_cast<size_t>(s) * d);
    for (size_t i = 0; i < kd.size(); ++i) {
        kd[i] = half_value(k[i]);
        vd[i] = half_value(v[i]);
    }
    std::vector<double> qrow(d), scores(s), rounded(s), acc(d);
    for (int row = row_begin; row < row_end; ++row) {
        for (int f = 0; f < d; ++f) qrow[f] = half_value(q[static_cast<size_t>(row) * d + f]);
        double maximum = -std::numeric_limits<double>::infinity();
        for (int t = 0; t < s; ++t) {
            double dot = 0.0;
            const double* kp = &kd[static_cast<size_t>(t) * d];
            for (int f = 0; f < d; ++f) dot += qrow[f] * kp[f];
            scores[t] = dot * scale;
            if ((!causal || t <= row) && scores[t] > maximum) maximum = scores[t];
        }
        double denominator = 0.0;
        for (int t = 0; t < s; ++t) {
            if (causal && t > row) {
                scores[t] = 0.0;
            } else {
                scores[t] = std::exp(scores[t] - maximum);
                denominator += scores[t];
            }
        }
        for (int t = 0; t < s; ++t) {
            const double p = scores[t] / denominator;
            if (prob) prob[static_cast<size_t>(row - row_begin) * s + t] = p;
            rounded[t] = half_value(to_half(p));
        }
        std::fill(acc.begin(), acc.end(), 0.0);
        for (int t = 0; t < s; ++t) {
            const double p = rounded[t];
            const double* vp = &vd[static_cast<size_t>(t) * d];
            for (int f = 0; f < d; ++f) acc[f] += p * vp[f];
        }
        for (int f = 0; f < d; ++f) out[static_cast<size_t>(row - row_begin) * d + f] = acc[f];
    }
}

// tests/attention_correctness.cu:19-21 and :172-177. The reference fixes s = 16
// and uses gamma(32); the general form uses gamma(2s).
void tko_attention_bound(const uint16_t* v, int s, int d, double* bound_per_col) {
    constexpr double eps = 0x1p-23;
    const double n = 2.0 * s;
    const double gamma = (n * eps) / (1.0 - n * eps);
    const double factor = 512.0 * eps + 0x1p-11 + gamma;
    for (int c = 0; c < d; ++c) {
        double scale = 0.0;
        for (int t = 0; t < s; ++t) scale += std::fabs(half_value(v[static_cast<size_t>(t) * d + c]));
        bound_per_col[c] = factor * scale;
    }
}

// Full-row softmax check: include/tk_sm7x/softmax.cuh:54-64 (exp(x - row max) /
// row sum) applied to rows of any length n instead of 16 columns, evaluated in
// FP64 from the FP32 inputs. Each element of `got` must be finite, in [0, 1] and
// within `bound` of the FP64 value, and each row of `got` must sum to 1 within
// `bound` (the checks of tests/tile_softmax.cu:160-173, row length generalised).
size_t tko_row_softmax_check(const float* x, size_t m, size_t n, size_t ldx, const float* got,
                             size_t ldg, double bound, double* max_err) {
    size_t failures = 0;
    double worst = 0.0;
    std::vector<double> e(n);
    for (size_t i = 0; i < m; ++i) {
        const float* row = x + i * ldx;
        const float* g = got + i * ldg;
        double maximum = -std::numeric_limits<double>::infinity();
        for (size_t c = 0; c < n; ++c) maximum = std::fmax(maximum, static_cast<double>(row[c]));
        double sum = 0.0;
        for (size_t c = 0; c < n; ++c) {
            e[c] = std::exp(static_cast<double>(row[c]) - maximum);
            sum += e[c];
        }
        double row_sum = 0.0;
        for (size_t c = 0; c < n; ++c) {
            const double want = e[c] / sum;
            const double err = std::fabs(static_cast<double>(g[c]) - want);
            if (std::isfinite(err) && err > worst) worst = err;
            if (!(std::isfinite(g[c]) && g[c] >= 0.0f && g[c] <= 1.0f && err <= bound)) ++failures;
            row_sum += static_cast<double>(g[c]);
        }
        if (!(std::fabs(row_sum - 1.0) <= bound)) ++failures;
    }
    if (max_err) *max_err = worst;
    return failures;
}

}  // extern "C"
