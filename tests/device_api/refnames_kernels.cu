// A user kernel written against the reference's device API names: it includes
// <tk_sm7x/reduce.cuh> and <tk_sm7x/softmax.cuh> and calls row_sum, row_max,
// row_softmax and row_softmax_causal with the reference's signatures
// (include/tk_sm7x/reduce.cuh:43-51, softmax.cuh:54-81 of ThunderKittens-SM7x):
// a shared st<float, 16, 16, row_major> staging tile, the accumulator tile rt_c,
// a scratch tile, 16-float row outputs. Only the source of rt_c differs from an
// SM7x kernel: load() from the staged tile instead of a warp-level mma().
// Compiled by tests/test_tile_api_gpu.py for sm_100a and driven through ctypes.
#include <cuda_runtime.h>

#include "tk_sm7x/reduce.cuh"
#include "tk_sm7x/softmax.cuh"

namespace {

constexpr int kWarps = 4;

__global__ void refnames_kernel(const float* tiles, int n_tiles, float* sums, float* maxs, float* soft,
                                float* causal) {
    __shared__ tk_sm7x::st<float, 16, 16, tk_sm7x::row_major> staged[kWarps];
    __shared__ tk_sm7x::st<float, 16, 16, tk_sm7x::row_major> probs[kWarps];
    __shared__ tk_sm7x::st<float, 16, 16, tk_sm7x::row_major> scratch[kWarps];
    const int w = static_cast<int>(threadIdx.x / 32);
    const int lane = static_cast<int>(threadIdx.x % 32);
    const int t = static_cast<int>(blockIdx.x) * kWarps + w;
    if (t >= n_tiles) return;  // warp-uniform
    for (int i = lane; i < 256; i += 32) staged[w].data[i] = tiles[static_cast<size_t>(t) * 256 + i];
    __syncwarp();
    tk_sm7x::rt_c c;
    tk_sm7x::load(c, staged[w]);
    tk_sm7x::row_sum(sums + static_cast<size_t>(t) * 16, c, scratch[w]);
    tk_sm7x::row_max(maxs + static_cast<size_t>(t) * 16, c, scratch[w]);
    tk_sm7x::row_softmax(probs[w], c, scratch[w]);
    for (int i = lane; i < 256; i += 32) soft[static_cast<size_t>(t) * 256 + i] = probs[w].data[i];
    __syncwarp();
    tk_sm7x::row_softmax_causal(probs[w], c, scratch[w]);
    for (int i = lane; i < 256; i += 32) causal[static_cast<size_t>(t) * 256 + i] = probs[w].data[i];
}

}  // namespace

extern "C" int refnames_run(const float* tiles, int n_tiles, float* sums, float* maxs, float* soft,
                            float* causal) {
    refnames_kernel<<<(n_tiles + kWarps - 1) / kWarps, kWarps * 32>>>(tiles, n_tiles, sums, maxs, soft, causal);
    if (cudaGetLastError() != cudaSuccess) return 1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}
