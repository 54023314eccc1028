// A caller written against ThunderKittens-SM7x's public headers, compiled unchanged
// against this repository's include/ and linked with libtk_b200.so. Exercises the
// GEMM and one-tile attention entry points with __half buffers and a
// non-blocking stream, and checks results that are exact for these inputs.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <vector>

#include "tk_sm7x/attention.cuh"
#include "tk_sm7x/gemm.cuh"
#include "tk_sm7x/reduce.cuh"
#include "tk_sm7x/softmax.cuh"

static int fail(const char* what) {
    std::fprintf(stderr, "FAIL: %s\n", what);
    return 1;
}

int main() {
    const int m = 32, n = 48, k = 32, lda = 37, ldb = 53, ldc = 59;
    std::vector<__half> a(m * lda), b(k * ldb);
    for (int r = 0; r < m; ++r)
        for (int c = 0; c < k; ++c) a[r * lda + c] = __float2half(static_cast<float>((r * 3 + c * 5) % 7 - 3));
    for (int r = 0; r < k; ++r)
        for (int c = 0; c < n; ++c) b[r * ldb + c] = __float2half(static_cast<float>((r * 2 + c * 3) % 5 - 2));
    __half *da, *db;
    float* dc;
    cudaMalloc(&da, a.size() * sizeof(__half));
    cudaMalloc(&db, b.size() * sizeof(__half));
    cudaMalloc(&dc, m * ldc * sizeof(float));
    cudaMemcpy(da, a.data(), a.size() * sizeof(__half), cudaMemcpyHostToDevice);
    cudaMemcpy(db, b.data(), b.size() * sizeof(__half), cudaMemcpyHostToDevice);
    std::vector<float> c(m * ldc, -123456.0f);
    cudaMemcpy(dc, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaStream_t stream;
    cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
    if (tk_sm7x::gemm_f16_f16_f32_nn(m, n, k, da, lda, db, ldb, dc, ldc, stream) != cudaSuccess)
        return fail("gemm launch");
    if (tk_sm7x::gemm_f16_f16_f32_nn(m, n, 17, da, lda, db, ldb, dc, ldc, stream) != cudaErrorInvalidValue)
        return fail("gemm invalid k");
    cudaStreamSynchronize(stream);
    cudaMemcpy(c.data(), dc, c.size() * sizeof(float), cudaMemcpyDeviceToHost);
    for (int r = 0; r < m; ++r) {
        for (int col = 0; col < n; ++col) {
            double want = 0;
            for (int kk = 0; kk < k; ++kk)
                want += static_cast<double>(__half2float(a[r * lda + kk])) * __half2float(b[kk * ldb + col]);
            if (c[r * ldc + col] != static_cast<float>(want)) return fail("gemm value");
        }
        for (int col = n; col < ldc; ++col)
            if (c[r * ldc + col] != -123456.0f) return fail("gemm padding");
    }
    // One-tile attention with uniform scores: P = 1/16 exactly, out = column means.
    std::vector<__half> q(256, __float2half(0.0f)), kv(256);
    for (int i = 0; i < 256; ++i) kv[i] = __float2half(static_cast<float>((i * 7) % 13 - 6) / 8.0f);
    __half *dq, *dk;
    float* dout;
    cudaMalloc(&dq, 512);
    cudaMalloc(&dk, 512);
    cudaMalloc(&dout, 1024);
    cudaMemcpy(dq, q.data(), 512, cudaMemcpyHostToDevice);
    cudaMemcpy(dk, kv.data(), 512, cudaMemcpyHostToDevice);
    if (tk_sm7x::attention_forward_16x16(dq, dk, dk, dout, stream) != cudaSuccess) return fail("attention");
    if (tk_sm7x::attention_forward_16x16(dq, nullptr, dk, dout, stream) != cudaErrorInvalidValue)
        return fail("attention null");
    std::vector<float> out(256);
    cudaStreamSynchronize(stream);
    cudaMemcpy(out.data(), dout, 1024, cudaMemcpyDeviceToHost);
    for (int r = 0; r < 16; ++r)
        for (int col = 0; col < 16; ++col) {
            double want = 0;
            for (int t = 0; t < 16; ++t) want += __half2float(kv[t * 16 + col]) / 16.0;
            if (out[r * 16 + col] != static_cast<float>(want)) return fail("attention value");
        }
    // Batched row reductions of the GEMM output's first 16x16 tile (as FP32 tiles).
    std::vector<float> tile(256);
    for (int i = 0; i < 256; ++i) tile[i] = static_cast<float>(i % 17) - 8.0f;
    float *dt, *ds;
    cudaMalloc(&dt, 1024);
    cudaMalloc(&ds, 1024);
    cudaMemcpy(dt, tile.data(), 1024, cudaMemcpyHostToDevice);
    if (tk_sm7x::tile_row_max(dt, 1, ds, stream) != cudaSuccess) return fail("row max");
    if (tk_sm7x::tile_row_softmax(dt, 1, dt, stream) != cudaSuccess) return fail("softmax in place");
    std::vector<float> mx(16);
    cudaStreamSynchronize(stream);
    cudaMemcpy(mx.data(), ds, 64, cudaMemcpyDeviceToHost);
    for (int r = 0; r < 16; ++r) {
        float want = tile[r * 16];
        for (int col = 1; col < 16; ++col) want = tile[r * 16 + col] > want ? tile[r * 16 + col] : want;
        if (mx[r] != want) return fail("row max value");
    }
    std::printf("drop-in: PASS\n");
    return 0;
}
