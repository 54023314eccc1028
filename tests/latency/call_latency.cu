// Per-call latency of the public entry points, measured from C++ the way
// ThunderKittens-SM7x's own benches measure them, so that no Python binding
// overhead enters the numbers:
//   * GEMM (bench/gemm_throughput.cu:94-120): two warm-up calls, then five calls
//     each bracketed by CUDA events on the default stream; the best one counts.
//     Square sizes 256..4096 and the decode shape 16 x 4096 x 4096.
//   * one-tile attention (bench/attention_throughput.cu:128-165, 206-233): 2048
//     back-to-back calls between two events, four rounds alternating unmasked and
//     causal, the median round in microseconds per public call.
// The library under test is libtk_b200.so (linked). When a path to the reference's
// own kernels built as compute_75 PTX (oracle/_ref/libtk_legacy.so) is given as
// argv[1], the same measurements run on it too, on the same GPU.
//
// Output: one JSON object per line, {"impl", "call", "us", "host_us"}; host_us is the
// CPU time spent inside the call itself (validation, descriptors, launch).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "tk_b200.h"

namespace {

using GemmFn = cudaError_t (*)(int, int, int, const void*, int, const void*, int, float*, int, cudaStream_t);
using AttnFn = cudaError_t (*)(const void*, const void*, const void*, float*, int, cudaStream_t);

struct Impl {
    const char* name;
    GemmFn gemm;
    AttnFn attention;  // (q, k, v, out, causal, stream)
};

cudaError_t ours_attention(const void* q, const void* k, const void* v, float* out, int causal,
                           cudaStream_t stream) {
    return causal ? tk_attention_forward_16x16_causal(q, k, v, out, stream)
                  : tk_attention_forward_16x16(q, k, v, out, stream);
}

bool check(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return true;
    std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(err));
    return false;
}

using Clock = std::chrono::steady_clock;

double since_us(Clock::time_point t0) {
    return std::chrono::duration<double, std::micro>(Clock::now() - t0).count();
}

// Best single-call time of an m x n x k GEMM (dense leading dimensions), in
// microseconds, and the smallest host time spent inside the call.
bool gemm_best_us(const Impl& impl, int m, int n, int k, const __half* a, const __half* b, float* c, double* us,
                  double* host_us) {
    for (int i = 0; i < 2; ++i)
        if (!check(impl.gemm(m, n, k, a, k, b, n, c, n, nullptr), "gemm warm-up")) return false;
    if (!check(cudaDeviceSynchronize(), "synchronize")) return false;
    cudaEvent_t start, stop;
    cudaEventCreate(&start);
    cudaEventCreate(&stop);
    float best = 0.0f;
    bool ok = true;
    *host_us = 1e30;
    for (int i = 0; i < 5 && ok; ++i) {
        ok = check(cudaEventRecord(start), "record");
        const Clock::time_point t0 = Clock::now();
        ok = ok && check(impl.gemm(m, n, k, a, k, b, n, c, n, nullptr), "gemm");
        *host_us = std::min(*host_us, since_us(t0));
        ok = ok && check(cudaEventRecord(stop), "record") && check(cudaEventSynchronize(stop), "sync");
        float ms = 0.0f;
        if (ok) cudaEventElapsedTime(&ms, start, stop);
        if (ok && (i == 0 || ms < best)) best = ms;
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    *us = 1e3 * best;
    return ok;
}

// Microseconds per call over `calls` back-to-back one-tile attention calls, and
// the host time per call of the same loop.
bool attention_round_us(const Impl& impl, int causal, const __half* q, float* out, int calls, double* us,
                        double* host_us) {
    for (int i = 0; i < 16; ++i)
        if (!check(impl.attention(q, q, q, out, causal, nullptr), "attention warm-up")) return false;
    if (!check(cudaDeviceSynchronize(), "synchronize")) return false;
    cudaEvent_t start, stop;
    cudaEventCreate(&start);
    cudaEventCreate(&stop);
    bool ok = check(cudaEventRecord(start), "record");
    const Clock::time_point t0 = Clock::now();
    for (int i = 0; i < calls && ok; ++i) ok = check(impl.attention(q, q, q, out, causal, nullptr), "attention");
    *host_us = since_us(t0) / calls;
    ok = ok && check(cudaEventRecord(stop), "record") && check(cudaEventSynchronize(stop), "sync");
    float ms = 0.0f;
    if (ok) cudaEventElapsedTime(&ms, start, stop);
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    *us = 1e3 * ms / calls;
    return ok;
}

}  // namespace

int main(int argc, char** argv) {
    std::vector<Impl> impls = {{"sm_100a", tk_gemm_f16_f16_f32_nn, ours_attention}};
    if (argc > 1) {
        void* handle = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
        if (handle == nullptr) {
            std::fprintf(stderr, "dlopen %s: %s\n", argv[1], dlerror());
            return 1;
        }
        impls.push_back({"legacy", reinterpret_cast<GemmFn>(dlsym(handle, "tkl_gemm_f16_f16_f32_nn")),
                         reinterpret_cast<AttnFn>(dlsym(handle, "tkl_attention_forward_16x16"))});
        if (impls.back().gemm == nullptr || impls.back().attention == nullptr) {
            std::fprintf(stderr, "legacy symbols missing\n");
            return 1;
        }
    }
    const int sizes[] = {256, 512, 1024, 2048, 4096};
    const size_t max_elems = 4096u * 4096u;
    __half *a = nullptr, *b = nullptr, *q = nullptr;
    float *c = nullptr, *out = nullptr;
    if (!check(cudaMalloc(&a, max_elems * 2), "malloc") || !check(cudaMalloc(&b, max_elems * 2), "malloc") ||
        !check(cudaMalloc(&c, max_elems * 4), "malloc") || !check(cudaMalloc(&q, 512), "malloc") ||
        !check(cudaMalloc(&out, 1024), "malloc"))
        return 1;
    // Inputs: small exact values (the timing does not depend on them).
    std::vector<__half> host(max_elems);
    for (size_t i = 0; i < max_elems; ++i) host[i] = __float2half(static_cast<float>(static_cast<int>(i % 7) - 3) / 4);
    cudaMemcpy(a, host.data(), max_elems * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(b, host.data(), max_elems * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(q, host.data(), 512, cudaMemcpyHostToDevice);

    for (const Impl& impl : impls) {
        for (int size : sizes) {
            double us = 0, host_us = 0;
            if (!gemm_best_us(impl, size, size, size, a, b, c, &us, &host_us)) return 1;
            std::printf("{\"impl\": \"%s\", \"call\": \"gemm_%d\", \"us\": %.3f, \"host_us\": %.3f}\n", impl.name,
                        size, us, host_us);
        }
        {
            // The decode-shaped configuration, 16 x 4096 x 4096.
            double us = 0, host_us = 0;
            if (!gemm_best_us(impl, 16, 4096, 4096, a, b, c, &us, &host_us)) return 1;
            std::printf("{\"impl\": \"%s\", \"call\": \"gemm_16x4096x4096\", \"us\": %.3f, \"host_us\": %.3f}\n",
                        impl.name, us, host_us);
        }
        double rounds[2][4], host[2][4];
        for (int round = 0; round < 4; ++round)
            for (int order = 0; order < 2; ++order) {
                const int causal = round % 2 == 0 ? order : 1 - order;
                if (!attention_round_us(impl, causal, q, out, 2048, &rounds[causal][round], &host[causal][round]))
                    return 1;
            }
        for (int causal = 0; causal < 2; ++causal) {
            std::sort(rounds[causal], rounds[causal] + 4);
            std::sort(host[causal], host[causal] + 4);
            std::printf("{\"impl\": \"%s\", \"call\": \"attention_16x16%s\", \"us\": %.3f, \"host_us\": %.3f}\n",
                        impl.name, causal ? "_causal" : "", (rounds[causal][1] + rounds[causal][2]) / 2,
                        (host[causal][1] + host[causal][2]) / 2);
        }
    }
    std::fflush(stdout);
    return 0;
}
