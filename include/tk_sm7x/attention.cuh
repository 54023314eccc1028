// Drop-in replacement for ThunderKittens-SM7x include/tk_sm7x/attention.cuh:15-23,
// plus the general [batch, heads, seq, head_dim] forward of the sm_100a library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#include "tk_b200.h"

namespace tk_sm7x {

// softmax(Q K^T / 4) V for one contiguous row-major 16x16 tile each; probabilities
// rounded to FP16 nearest-even before the PV product; FP32 out. Q, K, V may alias
// each other but not out. Null pointers return cudaErrorInvalidValue.
inline cudaError_t attention_forward_16x16(const __half* q, const __half* k, const __half* v,
                                           float* out, cudaStream_t stream = nullptr) {
    return tk_attention_forward_16x16(q, k, v, out, stream);
}

// Output row i attends only to key/value tokens 0..i.
inline cudaError_t attention_forward_16x16_causal(const __half* q, const __half* k,
                                                  const __half* v, float* out,
                                                  cudaStream_t stream = nullptr) {
    return tk_attention_forward_16x16_causal(q, k, v, out, stream);
}

// General forward, see tk_attention_forward_f16 in tk_b200.h.
inline cudaError_t attention_forward(const __half* q, const __half* k, const __half* v, float* out,
                                     int batch, int heads, int seq, int head_dim, float scale,
                                     bool causal, cudaStream_t stream = nullptr) {
    return tk_attention_forward_f16(q, k, v, out, batch, heads, seq, head_dim, scale,
                                    causal ? 1 : 0, stream);
}

}  // namespace tk_sm7x
