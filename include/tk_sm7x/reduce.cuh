// Row sums and maxima of 16x16 FP32 tiles: ThunderKittens-SM7x
// include/tk_sm7x/reduce.cuh:43-51, in two forms.
//
// Device (CUDA translation units): tk_sm7x::row_sum / row_max(float* dst,
// const rt_c& src, st<float, 16, 16, row_major>& scratch), the reference's
// signatures, with rt_c the sm_100a accumulator tile (tile_b200.cuh). Same call
// contract: all 32 lanes of a warp call convergently, dst holds 16 floats, the
// call ends with a warp barrier. The scratch tile is accepted for source
// compatibility and left untouched (the layout needs no shared-memory round trip).
//
// Host (batched): tile_row_sum / tile_row_max reduce n_tiles contiguous 16x16
// row-major FP32 tiles resident in device memory.
//
// Both use the reference's balanced column-order tree: bit-identical results, max
// ties (and signed zeros) pick the right operand.
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

#if defined(__CUDACC__)
#include "tk_sm7x/tile_b200.cuh"

namespace tk_sm7x {

__device__ __forceinline__ void row_sum(float* dst, const rt_c& src, st<float, 16, 16, row_major>& scratch) {
    static_cast<void>(scratch);
    b200::row_sum(dst, src);
}

__device__ __forceinline__ void row_max(float* dst, const rt_c& src, st<float, 16, 16, row_major>& scratch) {
    static_cast<void>(scratch);
    b200::row_max(dst, src);
}

}  // namespace tk_sm7x
#endif
