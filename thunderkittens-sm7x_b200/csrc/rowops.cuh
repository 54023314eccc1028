// rowops.cuh — batched 16x16 FP32 tile row operations (memory-bound).
//
// Replaces the warp-level row_sum / row_max / row_softmax / row_softmax_causal
// of ThunderKittens-SM7x (include/tk_sm7x/reduce.cuh:43-51,
// include/tk_sm7x/softmax.cuh:54-81) with batched kernels over tiles resident in
// HBM. Layout in HBM: tile t occupies floats [256 t, 256 t + 256), row-major.
//
// One warp owns one tile per step: lane l loads float4 number l (rows 0..7) and
// l + 32 (rows 8..15), so row r of a half-tile sits in lanes 4r..4r+3, lane 4r+j
// holding columns 4j..4j+3. Every warp load is a fully coalesced 512-byte run.
// The reduction tree is the reference's fixed balanced tree in column order
// (tests/row_reduce_reference.cuh:16-24): the lane-local ((c0 op c1) op (c2 op
// c3)) is the first two tree levels, then xor-1 and xor-2 shuffles combine
// lanes in order, the lower lane always supplying the left operand, so results
// are bit-identical to the reference tree (including max's signed-zero ties,
// include/tk_sm7x/row_reduce_ops.cuh:11-15).
#pragma once

#include "tk_ptx.cuh"
#include "tk_sm7x/tile_b200.cuh"

namespace tk {
namespace rowops {

enum : int { kSum = 1, kMax = 2, kSoftmax = 4, kCausal = 8 };

constexpr int kThreads = 256;            // 8 warps per block
constexpr int kTilesPerWarpStep = 8;     // tiles in flight per warp step (16 KiB of loads per warp)

// The tree, max-tie rule and softmax are the public device-level tile API
// (include/tk_sm7x/tile_b200.cuh), whose tile16 layout is exactly the layout of a
// warp's two float4 loads of a tile here.
using OpSum = tk_sm7x::b200::op_sum;
using OpMax = tk_sm7x::b200::op_max;
using tk_sm7x::b200::quad_softmax;

template <class Op>
__device__ __forceinline__ float quad_tree(float x0, float x1, float x2, float x3) {
    return tk_sm7x::b200::quad_reduce<Op>(x0, x1, x2, x3);
}

template <bool kVec>
__device__ __forceinline__ float4 load4(const float* p) {
    if constexpr (kVec) {
        return __ldcs(reinterpret_cast<const float4*>(p));
    } else {
        return make_float4(__ldcs(p), __ldcs(p + 1), __ldcs(p + 2), __ldcs(p + 3));
    }
}

template <bool kVec>
__device__ __forceinline__ void store4(float* p, float4 v) {
    if constexpr (kVec) {
        __stcs(reinterpret_cast<float4*>(p), v);
    } else {
        __stcs(p, v.x);
        __stcs(p + 1, v.y);
        __stcs(p + 2, v.z);
        __stcs(p + 3, v.w);
    }
}

template <int kOps, bool kVec>
__global__ void __launch_bounds__(kThreads) tile_row_ops_kernel(const float* tiles, size_t n_tiles,
                                                                float* sum_out, float* max_out,
                                                                float* softmax_out,
                                                                float* causal_out) {
    const unsigned lane = lane_id();
    const size_t warps_total = static_cast<size_t>(gridDim.x) * (kThreads / 32);
    const size_t warp_global = static_cast<size_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
    const int quad_row = static_cast<int>(lane >> 2);  // row within a half-tile

    for (size_t first = warp_global * kTilesPerWarpStep; first < n_tiles;
         first += warps_total * kTilesPerWarpStep) {
        float4 v[kTilesPerWarpStep][2];
#pragma unroll
        for (int u = 0; u < kTilesPerWarpStep; ++u) {
            const size_t t = first + u;
            if (t < n_tiles) {
                const float* base = tiles + t * 256;
                v[u][0] = load4<kVec>(base + lane * 4);
                v[u][1] = load4<kVec>(base + 128 + lane * 4);
            } else {
                v[u][0] = v[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < kTilesPerWarpStep; ++u) {
            const size_t t = first + u;
            if (t >= n_tiles) continue;  // warp-uniform
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float4 x = v[u][h];
                const int row = h * 8 + quad_row;
                if constexpr ((kOps & kSum) != 0) {
                    const float s = quad_tree<OpSum>(x.x, x.y, x.z, x.w);
                    if ((lane & 3u) == 0) __stcs(sum_out + t * 16 + row, s);
                }
                if constexpr ((kOps & kMax) != 0) {
                    const float m = quad_tree<OpMax>(x.x, x.y, x.z, x.w);
                    if ((lane & 3u) == 0) __stcs(max_out + t * 16 + row, m);
                }
                if constexpr ((kOps & kSoftmax) != 0) {
                    store4<kVec>(softmax_out + t * 256 + h * 128 + lane * 4, quad_softmax<false>(x, row));
                }
                if constexpr ((kOps & kCausal) != 0) {
                    store4<kVec>(causal_out + t * 256 + h * 128 + lane * 4, quad_softmax<true>(x, row));
                }
            }
        }
    }
}

}  // namespace rowops
}  // namespace tk
