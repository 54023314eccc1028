// tile_b200.cuh — device-level 16x16 FP32 tile row operations for sm_100a
// kernels (header only; include from .cu files compiled for sm_100a).
//
// The sm_100a counterpart of ThunderKittens-SM7x's warp tile API
// (include/tk_sm7x/reduce.cuh:43-51, include/tk_sm7x/softmax.cuh:54-81). The
// reference keeps a 16x16 accumulator in an SM7x MMA fragment (rt_c); tcgen05 has
// no warp-sized 16x16 MMA, so here a warp holds a 16x16 tile in a fixed, documented
// register layout instead:
//
//   tile16: lane l holds row l/4, columns 4*(l%4) .. 4*(l%4)+3 in `lo`, and
//           row 8 + l/4, same columns, in `hi`.
//
// That is the layout of two coalesced 512-byte float4 loads of a row-major tile,
// and the layout the library's batched row-op kernels use. Reductions follow the
// reference's fixed balanced column-order tree (tests/row_reduce_reference.cuh:
// 16-24): the lane-local ((c0 op c1) op (c2 op c3)) are the first two levels and
// ordered xor-shuffles the last two, the lower lane always the left operand, so
// sums and maxima are bit-identical to the reference tree, signed-zero max ties
// included (include/tk_sm7x/row_reduce_ops.cuh:11-15).
//
// For epilogues that hold one row per thread (the layout tcgen05.ld 32x32b gives),
// row_tree16_sum / row_tree16_max reduce 16 consecutive values of one row with the
// same tree.
//
// All tile16 functions are warp-collective: all 32 lanes call them convergently.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace tk_sm7x {
namespace b200 {

struct tile16 {
    float4 lo;  // row lane/4
    float4 hi;  // row 8 + lane/4
};

struct op_sum {
    __device__ __forceinline__ static float apply(float low, float high) { return low + high; }
};

// Ties (and signed zeros) pick the right operand, as row_reduce_ops.cuh:11-15.
struct op_max {
    __device__ __forceinline__ static float apply(float low, float high) {
        return low > high ? low : high;
    }
};

__device__ __forceinline__ unsigned tile_lane() { return threadIdx.x & 31u; }

// Balanced 16-column tree for the row whose four columns groups sit in the lane's
// quad (lanes 4r..4r+3); every lane of the quad gets the result.
template <class Op>
__device__ __forceinline__ float quad_reduce(float x0, float x1, float x2, float x3) {
    const unsigned j = tile_lane() & 3u;
    float v = Op::apply(Op::apply(x0, x1), Op::apply(x2, x3));
    float o = __shfl_xor_sync(0xffffffffu, v, 1);
    v = (j & 1u) ? Op::apply(o, v) : Op::apply(v, o);
    o = __shfl_xor_sync(0xffffffffu, v, 2);
    v = (j & 2u) ? Op::apply(o, v) : Op::apply(v, o);
    return v;
}

// Canonical tree over 16 consecutive values held by one thread.
template <class Op>
__device__ __forceinline__ float tree16(const float* x) {
    const float q0 = Op::apply(Op::apply(x[0], x[1]), Op::apply(x[2], x[3]));
    const float q1 = Op::apply(Op::apply(x[4], x[5]), Op::apply(x[6], x[7]));
    const float q2 = Op::apply(Op::apply(x[8], x[9]), Op::apply(x[10], x[11]));
    const float q3 = Op::apply(Op::apply(x[12], x[13]), Op::apply(x[14], x[15]));
    return Op::apply(Op::apply(q0, q1), Op::apply(q2, q3));
}

__device__ __forceinline__ float row_tree16_sum(const float* x16) { return tree16<op_sum>(x16); }
__device__ __forceinline__ float row_tree16_max(const float* x16) { return tree16<op_max>(x16); }

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Softmax of the row held by the lane's quad; `row` is the tile row, the lane holds
// columns 4j..4j+3 (j = lane % 4). Causal: columns > row take no part in the max
// and sum and come out as exactly +0 (softmax.cuh:69-81). The max and sum use the
// balanced tree; exp(x - m) is 2^((x - m) log2 e) on the MUFU unit and the
// normalisation one correctly rounded reciprocal per row times each exponential,
// within ~2e-6 of the FP64 softmax (the reference's bound is 512 * 2^-23).
template <bool kCausal>
__device__ __forceinline__ float4 quad_softmax(float4 v, int row) {
    constexpr float kLog2e = 1.4426950408889634f;
    const int c0 = static_cast<int>(tile_lane() & 3u) * 4;
    if constexpr (kCausal) {
        if (c0 + 0 > row) v.x = -INFINITY;
        if (c0 + 1 > row) v.y = -INFINITY;
        if (c0 + 2 > row) v.z = -INFINITY;
        if (c0 + 3 > row) v.w = -INFINITY;
    }
    const float m = quad_reduce<op_max>(v.x, v.y, v.z, v.w);
    float4 e;
    e.x = ex2_approx((v.x - m) * kLog2e);  // masked: 2^-inf = +0 exactly
    e.y = ex2_approx((v.y - m) * kLog2e);
    e.z = ex2_approx((v.z - m) * kLog2e);
    e.w = ex2_approx((v.w - m) * kLog2e);
    const float s = quad_reduce<op_sum>(e.x, e.y, e.z, e.w);
    const float inv = __frcp_rn(s);
    return make_float4(e.x * inv, e.y * inv, e.z * inv, e.w * inv);
}

// Loads a row-major 16x16 tile (leading dimension ld floats) from shared or
// global memory. Rows that are 16-byte aligned use float4 accesses.
__device__ __forceinline__ void load(tile16& t, const float* src, int ld) {
    const unsigned lane = tile_lane();
    const float* p0 = src + static_cast<size_t>(lane >> 2) * ld + (lane & 3u) * 4;
    const float* p1 = p0 + static_cast<size_t>(8) * ld;
    if ((ld & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        t.lo = *reinterpret_cast<const float4*>(p0);
        t.hi = *reinterpret_cast<const float4*>(p1);
    } else {
        t.lo = make_float4(p0[0], p0[1], p0[2], p0[3]);
        t.hi = make_float4(p1[0], p1[1], p1[2], p1[3]);
    }
}

__device__ __forceinline__ void store(float* dst, int ld, const tile16& t) {
    const unsigned lane = tile_lane();
    float* p0 = dst + static_cast<size_t>(lane >> 2) * ld + (lane & 3u) * 4;
    float* p1 = p0 + static_cast<size_t>(8) * ld;
    if ((ld & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        *reinterpret_cast<float4*>(p0) = t.lo;
        *reinterpret_cast<float4*>(p1) = t.hi;
    } else {
        p0[0] = t.lo.x; p0[1] = t.lo.y; p0[2] = t.lo.z; p0[3] = t.lo.w;
        p1[0] = t.hi.x; p1[1] = t.hi.y; p1[2] = t.hi.z; p1[3] = t.hi.w;
    }
}

// Element-wise in registers: the counterparts of tk_sm7x::zero / tk_sm7x::scale
// (include/tk_sm7x/tile.cuh:126-153). Scaling is one FP32 multiply per element,
// exact for power-of-two factors in the normal range.
__device__ __forceinline__ void zero(tile16& t) {
    t.lo = make_float4(0.f, 0.f, 0.f, 0.f);
    t.hi = make_float4(0.f, 0.f, 0.f, 0.f);
}

__device__ __forceinline__ void scale(tile16& t, float factor) {
    t.lo.x *= factor;
    t.lo.y *= factor;
    t.lo.z *= factor;
    t.lo.w *= factor;
    t.hi.x *= factor;
    t.hi.y *= factor;
    t.hi.z *= factor;
    t.hi.w *= factor;
}

// Row sums / maxima in registers: .x is the lane's row lane/4, .y row 8 + lane/4.
__device__ __forceinline__ float2 row_sum(const tile16& t) {
    return make_float2(quad_reduce<op_sum>(t.lo.x, t.lo.y, t.lo.z, t.lo.w),
                       quad_reduce<op_sum>(t.hi.x, t.hi.y, t.hi.z, t.hi.w));
}

__device__ __forceinline__ float2 row_max(const tile16& t) {
    return make_float2(quad_reduce<op_max>(t.lo.x, t.lo.y, t.lo.z, t.lo.w),
                       quad_reduce<op_max>(t.hi.x, t.hi.y, t.hi.z, t.hi.w));
}

// The same, written to dst[0..15] in row order (shared or global memory). Ends
// with a warp barrier, so the warp may read dst on return (reduce.cuh:12-19).
__device__ __forceinline__ void row_sum(float* dst, const tile16& t) {
    const float2 s = row_sum(t);
    const unsigned lane = tile_lane();
    if ((lane & 3u) == 0) {
        dst[lane >> 2] = s.x;
        dst[8 + (lane >> 2)] = s.y;
    }
    __syncwarp();
}

__device__ __forceinline__ void row_max(float* dst, const tile16& t) {
    const float2 m = row_max(t);
    const unsigned lane = tile_lane();
    if ((lane & 3u) == 0) {
        dst[lane >> 2] = m.x;
        dst[8 + (lane >> 2)] = m.y;
    }
    __syncwarp();
}

// Row softmax of a tile, in registers; the source tile is unchanged.
__device__ __forceinline__ tile16 row_softmax(const tile16& t) {
    const int r = static_cast<int>(tile_lane() >> 2);
    return tile16{quad_softmax<false>(t.lo, r), quad_softmax<false>(t.hi, r + 8)};
}

// Row i uses columns 0..i; the others are exactly 0.
__device__ __forceinline__ tile16 row_softmax_causal(const tile16& t) {
    const int r = static_cast<int>(tile_lane() >> 2);
    return tile16{quad_softmax<true>(t.lo, r), quad_softmax<true>(t.hi, r + 8)};
}

}  // namespace b200

// Reference-named tile types, so that device code written against the reference's
// warp tile API (include/tk_sm7x/tile.cuh:30-70) keeps its declarations:
//   st<T, R, C, Layout>  shared-memory tile: R x C elements in `data`, 32-byte aligned
//                        (the reference's tile.cuh:30-52 type; row- or column-major);
//   rt_c                 the 16x16 FP32 accumulator tile a warp holds. On sm_100a it
//                        is b200::tile16 (documented register layout above) instead
//                        of an SM7x MMA fragment; it is filled by load() from a
//                        shared or global tile rather than by a warp-level mma().
struct row_major {};
struct col_major {};

template <class T, int R, int C, class Layout = row_major>
struct alignas(32) st {
    T data[static_cast<size_t>(R) * C];
};

using rt_c = b200::tile16;

// Shared tile <-> accumulator tile (warp-collective, row-major FP32 tiles).
__device__ __forceinline__ void load(rt_c& dst, const st<float, 16, 16, row_major>& src) {
    b200::load(dst, src.data, 16);
}

__device__ __forceinline__ void store(st<float, 16, 16, row_major>& dst, const rt_c& src) {
    b200::store(dst.data, 16, src);
}

__device__ __forceinline__ void zero(rt_c& t) { b200::zero(t); }
__device__ __forceinline__ void scale(rt_c& t, float factor) { b200::scale(t, factor); }

}  // namespace tk_sm7x
