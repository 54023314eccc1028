// Exposes the reference's numerical bound helpers (tests/numerical_bounds.hpp)
// through a C ABI so the restated oracle can be checked against them. Built
// only from the reference sources where they lie; output goes to oracle/_ref/.
#include "numerical_bounds.hpp"

extern "C" double tkref_error_bound(int k, double sum_abs) {
    return tk_sm7x::test::numerical::error_bound(k, sum_abs);
}

extern "C" int tkref_within_bound(double actual, double reference, double bound) {
    return tk_sm7x::test::numerical::within_bound(actual, reference, bound) ? 1 : 0;
}
