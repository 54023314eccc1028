// A user kernel built on the device-level tile API (include/tk_sm7x/tile_b200.cuh),
// compiled by tests/test_tile_api_gpu.py for sm_100a and driven through ctypes.
// One warp per 16x16 tile: load (any leading dimension), the memory and register
// forms of row_sum / row_max, row_softmax, row_softmax_causal, and the
// thread-per-row tree.
#include <cuda_runtime.h>

#include "tk_sm7x/tile_b200.cuh"

namespace b200 = tk_sm7x::b200;

__global__ void tile_api_kernel(const float* in, int ld, int n_tiles, float* sums, float* maxs,
                                float* reg_sums, float* reg_maxs, float* tree_sums, float* softmax,
                                float* causal) {
    const int warps = blockDim.x / 32;
    const int t = blockIdx.x * warps + threadIdx.x / 32;
    if (t >= n_tiles) return;  // warp-uniform
    const float* src = in + static_cast<size_t>(t) * 16 * ld;
    b200::tile16 tile;
    b200::load(tile, src, ld);
    b200::row_sum(sums + t * 16, tile);
    b200::row_max(maxs + t * 16, tile);
    const float2 s = b200::row_sum(tile);
    const float2 m = b200::row_max(tile);
    const unsigned lane = threadIdx.x & 31u;
    if ((lane & 3u) == 1) {  // any lane of the quad holds the row's value
        reg_sums[t * 16 + (lane >> 2)] = s.x;
        reg_sums[t * 16 + 8 + (lane >> 2)] = s.y;
        reg_maxs[t * 16 + (lane >> 2)] = m.x;
        reg_maxs[t * 16 + 8 + (lane >> 2)] = m.y;
    }
    if (lane < 16) {
        float row[16];
        for (int c = 0; c < 16; ++c) row[c] = src[lane * ld + c];
        tree_sums[t * 16 + lane] = b200::row_tree16_sum(row);
    }
    b200::store(softmax + static_cast<size_t>(t) * 256, 16, b200::row_softmax(tile));
    b200::store(causal + static_cast<size_t>(t) * 256, 16, b200::row_softmax_causal(tile));
}

extern "C" int tile_api_run(const float* in, int ld, int n_tiles, float* sums, float* maxs,
                            float* reg_sums, float* reg_maxs, float* tree_sums, float* softmax,
                            float* causal) {
    const int warps = 4;
    tile_api_kernel<<<(n_tiles + warps - 1) / warps, warps * 32>>>(in, ld, n_tiles, sums, maxs, reg_sums,
                                                                   reg_maxs, tree_sums, softmax, causal);
    if (cudaGetLastError() != cudaSuccess) return 1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}

// tk_sm7x::scale's counterpart: load a tile, scale it in registers, store it.
__global__ void tile_scale_kernel(const float* in, float* out, float factor) {
    b200::tile16 tile;
    b200::load(tile, in, 16);
    b200::scale(tile, factor);
    b200::store(out, 16, tile);
}

extern "C" int tile_scale_run(const float* in, float* out, float factor) {
    tile_scale_kernel<<<1, 32>>>(in, out, factor);
    if (cudaGetLastError() != cudaSuccess) return 1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}
