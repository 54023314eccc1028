// Drop-in replacement for ThunderKittens-SM7x include/tk_sm7x/gemm.cuh:15-20.
// Same name, signature, default stream argument and contract; the work is done by
// the sm_100a library (link with libtk_b200.so, include <repo>/include).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#include "tk_b200.h"

namespace tk_sm7x {

// A is m-by-k, B is k-by-n, C is m-by-n; non-overlapping row-major device buffers.
// m, n, k positive multiples of 16; lda >= k, ldb >= n, ldc >= n. Returns
// cudaErrorInvalidValue without launching (and without touching the pending
// error) on invalid arguments; otherwise clears the pending error, enqueues on
// `stream` and returns cudaGetLastError().
inline cudaError_t gemm_f16_f16_f32_nn(int m, int n, int k, const __half* a, int lda,
                                       const __half* b, int ldb, float* c, int ldc,
                                       cudaStream_t stream = nullptr) {
    return tk_gemm_f16_f16_f32_nn(m, n, k, a, lda, b, ldb, c, ldc, stream);
}

}  // namespace tk_sm7x
