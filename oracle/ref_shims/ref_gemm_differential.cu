// Exposes the host fixture generators and FP64 reference of the reference's
// tests/gemm_differential.cu (fill_inputs :263-308, make_reference :380-401)
// through a C ABI. The test file is compiled as-is from the reference tree;
// its main() is renamed so this translation unit can be a shared library.
#include <cstdint>
#include <cstring>
#define main tkref_gemm_differential_main
#include "gemm_differential.cu"
#undef main

namespace {
GemmCase make_case(int m, int n, int k, int lda, int ldb, int ldc, int pattern) {
    return GemmCase{"golden", m, n, k, lda, ldb, ldc, static_cast<Pattern>(pattern)};
}
}  // namespace

extern "C" int tkref_diff_model_case_count() {
    return static_cast<int>(sizeof(kModelCases) / sizeof(kModelCases[0]));
}

// dims receives m, n, k, lda, ldb, ldc, pattern.
extern "C" const char* tkref_diff_model_case(int index, int* dims) {
    const GemmCase& c = kModelCases[index];
    dims[0] = c.m; dims[1] = c.n; dims[2] = c.k;
    dims[3] = c.lda; dims[4] = c.ldb; dims[5] = c.ldc;
    dims[6] = static_cast<int>(c.pattern);
    return c.name;
}

extern "C" void tkref_diff_fill(int m, int n, int k, int lda, int ldb, int ldc,
                                int pattern, uint16_t* a, uint16_t* b) {
    const GemmCase c = make_case(m, n, k, lda, ldb, ldc, pattern);
    std::vector<__half> va(static_cast<std::size_t>(m) * lda);
    std::vector<__half> vb(static_cast<std::size_t>(k) * ldb);
    fill_inputs(c, &va, &vb);
    std::memcpy(a, va.data(), va.size() * sizeof(__half));
    std::memcpy(b, vb.data(), vb.size() * sizeof(__half));
}

// value/sum_abs/bound each hold m * ldc doubles (padding cells keep the
// reference's NaN / 0 / 0 initialisation).
extern "C" void tkref_diff_reference(int m, int n, int k, int lda, int ldb, int ldc,
                                     int pattern, int model, const uint16_t* a,
                                     const uint16_t* b, double* value,
                                     double* sum_abs, double* bound) {
    const GemmCase c = make_case(m, n, k, lda, ldb, ldc, pattern);
    std::vector<__half> va(static_cast<std::size_t>(m) * lda);
    std::vector<__half> vb(static_cast<std::size_t>(k) * ldb);
    std::memcpy(va.data(), a, va.size() * sizeof(__half));
    std::memcpy(vb.data(), b, vb.size() * sizeof(__half));
    const std::vector<ReferenceCell> ref =
        make_reference(c, va, vb, model ? ComparisonMode::model : ComparisonMode::exact);
    for (std::size_t i = 0; i < ref.size(); ++i) {
        value[i] = ref[i].value;
        sum_abs[i] = ref[i].sum_abs;
        bound[i] = ref[i].bound;
    }
}
