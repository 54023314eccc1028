// Exposes fill_inputs (:52-89, seeded std::mt19937 uniform inputs and the
// identity/fingerprint patterns) and make_reference (:91-116) of the
// reference's tests/gemm_correctness.cu through a C ABI.
#include <cstdint>
#include <cstring>
#define main tkref_gemm_correctness_main
#include "gemm_correctness.cu"
#undef main

namespace {
GemmCase make_case(int m, int n, int k, int lda, int ldb, int ldc, int pattern,
                   unsigned seed) {
    return GemmCase{"golden", m, n, k, lda, ldb, ldc, static_cast<Pattern>(pattern),
                    seed, false, false};
}
}  // namespace

extern "C" void tkref_corr_fill(int m, int n, int k, int lda, int ldb, int ldc,
                                int pattern, unsigned seed, uint16_t* a, uint16_t* b) {
    const GemmCase c = make_case(m, n, k, lda, ldb, ldc, pattern, seed);
    std::vector<__half> va(static_cast<std::size_t>(m) * lda);
    std::vector<__half> vb(static_cast<std::size_t>(k) * ldb);
    fill_inputs(c, &va, &vb);
    std::memcpy(a, va.data(), va.size() * sizeof(__half));
    std::memcpy(b, vb.data(), vb.size() * sizeof(__half));
}

// out holds m * ldc floats; padding keeps the reference's sentinel.
extern "C" void tkref_corr_reference(int m, int n, int k, int lda, int ldb, int ldc,
                                     int pattern, unsigned seed, const uint16_t* a,
                                     const uint16_t* b, float* out) {
    const GemmCase c = make_case(m, n, k, lda, ldb, ldc, pattern, seed);
    std::vector<__half> va(static_cast<std::size_t>(m) * lda);
    std::vector<__half> vb(static_cast<std::size_t>(k) * ldb);
    std::memcpy(va.data(), a, va.size() * sizeof(__half));
    std::memcpy(vb.data(), b, vb.size() * sizeof(__half));
    const std::vector<float> ref = make_reference(c, va, vb);
    std::memcpy(out, ref.data(), ref.size() * sizeof(float));
}

extern "C" float tkref_corr_sentinel() { return kSentinel; }
