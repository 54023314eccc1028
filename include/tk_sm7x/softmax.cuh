// Row softmax of 16x16 FP32 tiles (and the causal-prefix variant): ThunderKittens-SM7x
// include/tk_sm7x/softmax.cuh:54-81, in two forms.
//
// Device (CUDA translation units): tk_sm7x::row_softmax / row_softmax_causal(
// st<float, 16, 16, row_major>& dst, const rt_c& logits, st<...>& scratch), the
// reference's signatures with rt_c the sm_100a accumulator tile (tile_b200.cuh).
// All 32 lanes of a warp call convergently; dst receives the probabilities row
// by row and the call ends with a warp barrier, so the warp may read dst on
// return; the logits are unchanged and scratch is left untouched.
//
// Host (batched): tile_row_softmax / tile_row_softmax_causal over n_tiles
// contiguous tiles in device memory, 256 output floats per tile.
//
// Row i of the causal form uses columns 0..i; columns after i are exactly 0.
// Probabilities are within 512 * 2^-23 of the FP64 softmax (tests/tile_softmax.cu:20).
#pragma once

#include <cstddef>

#include <cuda_runtime_api.h>

#include "tk_b200.h"

namespace tk_sm7x {

inline cudaError_t tile_row_softmax(const float* tiles, std::size_t n_tiles, float* out,
                                    cudaStream_t stream = nullptr) {
    return tk_tile_row_softmax_f32(tiles, n_tiles, out, stream);
}

// Row i uses columns 0..i; columns after i are exactly 0.
inline cudaError_t tile_row_softmax_causal(const float* tiles, std::size_t n_tiles, float* out,
                                           cudaStream_t stream = nullptr) {
    return tk_tile_row_softmax_causal_f32(tiles, n_tiles, out, stream);
}

}  // namespace tk_sm7x

#if defined(__CUDACC__)
#include "tk_sm7x/tile_b200.cuh"

namespace tk_sm7x {

__device__ __forceinline__ void row_softmax(st<float, 16, 16, row_major>& dst, const rt_c& logits,
                                            st<float, 16, 16, row_major>& scratch) {
    static_cast<void>(scratch);
    store(dst, b200::row_softmax(logits));
    __syncwarp();
}

__device__ __forceinline__ void row_softmax_causal(st<float, 16, 16, row_major>& dst, const rt_c& logits,
                                                   st<float, 16, 16, row_major>& scratch) {
    static_cast<void>(scratch);
    store(dst, b200::row_softmax_causal(logits));
    __syncwarp();
}

}  // namespace tk_sm7x
#endif
