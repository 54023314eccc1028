// Exposes the canonical row tree and 2Sum census of the reference's
// tests/row_reduce_reference.cuh (:16-54) and the seeded fixture values of
// tests/row_reduce.cu (:148-176) through a C ABI.
#include <cstdint>
#include <cstring>
#define main tkref_row_reduce_main
#include "row_reduce.cu"
#undef main

extern "C" float tkref_canonical_row(const float* row, int op) {
    if (op == 0) return tk_sm7x::test::canonical_row<tk_sm7x::detail::row_sum_op>(row);
    return tk_sm7x::test::canonical_row<tk_sm7x::detail::row_max_op>(row);
}

extern "C" int tkref_rounding_census(const float* row) {
    tk_sm7x::test::rounding_census_combine census;
    tk_sm7x::test::canonical_row_tree(census, row);
    return census.inexact;
}

extern "C" uint16_t tkref_row_exact_value(int row, int col, int seed) {
    const __half h = exact_value(row, col, seed);
    uint16_t bits;
    std::memcpy(&bits, &h, sizeof(bits));
    return bits;
}

extern "C" uint16_t tkref_row_rounded_value(int row, int col, uint32_t seed) {
    const __half h = rounded_value(fingerprint(row, col, seed));
    uint16_t bits;
    std::memcpy(&bits, &h, sizeof(bits));
    return bits;
}
