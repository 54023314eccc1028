// Batched host counterparts of ThunderKittens-SM7x include/tk_sm7x/reduce.cuh:43-51.
// The reference's row_sum / row_max reduce one 16x16 FP32 accumulator held by a
// warp; here they reduce n_tiles contiguous 16x16 row-major FP32 tiles resident in
// device memory, with the same balanced column-order tree (bit-identical results;
// max ties pick the right operand).
#pragma once

#include <cstddef>

#include <cuda_runtime_api.h>

#include "tk_b200.h"

namespace tk_sm7x {

inline cudaError_t tile_row_sum(const float* tiles, std::size_t n_tiles, float* out,
                                cudaStream_t stream = nullptr) {
    return tk_tile_row_sum_f32(tiles, n_tiles, out, stream);
}

inline cudaError_t tile_row_max(const float* tiles, std::size_t n_tiles, float* out,
                                cudaStream_t stream = nullptr) {
    return tk_tile_row_max_f32(tiles, n_tiles, out, stream);
}

}  // namespace tk_sm7x
