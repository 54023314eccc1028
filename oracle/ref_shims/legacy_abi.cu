// Legacy-path comparison harness (test and measurement infrastructure, never the
// product path): C entry points over ThunderKittens-SM7x's own
// tk_sm7x::gemm_f16_f16_f32_nn (src/gemm.cu:184-206) and
// tk_sm7x::attention_forward_16x16[_causal] (src/attention.cu:76-86), compiled
// from the reference sources as compute_75 PTX only, so the CUDA driver
// JIT-compiles the reference's WMMA kernels for whatever GPU runs them. On a B200
// this is "the legacy SM7x path on the same box", not a Blackwell implementation.
#include <cuda_fp16.h>

#include "tk_sm7x/attention.cuh"
#include "tk_sm7x/gemm.cuh"

extern "C" cudaError_t tkl_gemm_f16_f16_f32_nn(int m, int n, int k, const void* a, int lda, const void* b,
                                              int ldb, float* c, int ldc, cudaStream_t stream) {
    return tk_sm7x::gemm_f16_f16_f32_nn(m, n, k, static_cast<const __half*>(a), lda,
                                        static_cast<const __half*>(b), ldb, c, ldc, stream);
}

extern "C" cudaError_t tkl_attention_forward_16x16(const void* q, const void* k, const void* v, float* out,
                                                  int causal, cudaStream_t stream) {
    const __half* hq = static_cast<const __half*>(q);
    const __half* hk = static_cast<const __half*>(k);
    const __half* hv = static_cast<const __half*>(v);
    return causal ? tk_sm7x::attention_forward_16x16_causal(hq, hk, hv, out, stream)
                  : tk_sm7x::attention_forward_16x16(hq, hk, hv, out, stream);
}
