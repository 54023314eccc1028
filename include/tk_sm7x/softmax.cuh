// Batched host counterparts of ThunderKittens-SM7x include/tk_sm7x/softmax.cuh:54-81:
// per-row softmax (and the causal-prefix variant) of n_tiles contiguous 16x16
// row-major FP32 tiles in device memory, 256 output floats per tile.
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
