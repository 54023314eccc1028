// Cycles per tcgen05.mma (kind::f16, FP32 accumulate, M = 128, cta_group::1)
// issued back to back by one thread, for the operand shapes the attention and
// GEMM kernels use. Each case issues 256 groups of 8 MMAs (K = 16 each) and
// times them with clock64 up to the completion of the last one. "reused": every
// group reads the same shared-memory B tile; "fresh": consecutive groups read
// different B tiles, as the attention kernel's S = Q K^T (SS, K-major B) and
// O += P V (TS: P in tensor memory, MN-major B) groups do. Inputs are zero; only
// the timing is of interest. Output: one JSON object per line.
#include <cuda_fp16.h>

#include <cstdio>

#include "tk_ptx.cuh"

using namespace tk;

namespace {

constexpr int kGroups = 256;
constexpr int kSmemBytes = 96 * 1024 + 2048;

enum Case : int {
    kSsN128Reused,
    kSsN128Fresh,
    kTsN128Reused,
    kTsN128Fresh,
    kSsN256Reused,
    kSsN256Fresh,
    kAttentionOrder,  // S0, PV1, S1, PV0 groups on two K and two V tiles
    kTsAltMajor,      // all TS: S-style (A = Q in TMEM, B K-major) / PV-style (B MN-major) groups
    kTsAltSameDesc,   // all TS, both B K-major (one instruction descriptor)
    kSsAltMajor,      // all SS: B K-major / MN-major groups
    kTsAltNoHazard,   // all TS, one descriptor, alternating A and D regions that never overlap
    kSsDEachGroup,    // SS, accumulator region switched every group
    kTsAltMajorNoHazard,  // all TS, no TMEM overlap, odd groups with an MN-major B (another descriptor)
    kCases
};

template <int kCase>
__global__ void __launch_bounds__(128, 1) mma_rate(unsigned long long* cycles) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    // A: 32 KiB at base; B: two 32 KiB tiles at base + 32 KiB and base + 64 KiB.
    for (int i = threadIdx.x; i < (96 * 1024) / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    const uint32_t a_addr = base, b_addr = base + 32768;
    const uint32_t bar = base + 98304;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 98304 + 64);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 32) {
        tmem_alloc<1>(smem_u32(slot), 512);
        tmem_relinquish<1>();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *slot;
    if (threadIdx.x == 0) {
        constexpr uint32_t kIdS = idesc_f16_f32(128, 128, 0, 0);   // B K-major
        constexpr uint32_t kIdO = idesc_f16_f32(128, 128, 0, 1);   // B MN-major
        constexpr uint32_t kIdW = idesc_f16_f32(128, 256, 0, 0);   // N = 256
        const unsigned long long t0 = clock64();
        for (int g = 0; g < kGroups; ++g) {
            const uint32_t b_tile = (kCase == kSsN128Reused || kCase == kTsN128Reused || kCase == kSsN256Reused)
                                        ? 0u
                                        : static_cast<uint32_t>(g & 1) * 32768u;
            const uint32_t which = static_cast<uint32_t>(g >> 1) & 1u;
            const bool pv = kCase == kTsN128Reused || kCase == kTsN128Fresh || (kCase == kAttentionOrder && (g & 1));
            const bool odd = (g & 1) != 0;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                if (kCase == kTsAltMajorNoHazard) {
                    if (!odd)
                        mma_f16_ts(tmem + 64u, tmem + kk * 8, sw128_desc(b_addr + off, 16, 1024), kIdS,
                                   kk > 0 ? 1u : 0u);
                    else
                        mma_f16_ts(tmem + 192u, tmem + 448u + kk * 8,
                                   sw128_desc(b_addr + 32768 + kk * 2048, 16384, 1024), kIdO, kk > 0 ? 1u : 0u);
                } else if (kCase == kTsAltNoHazard) {
                    // even: A [0,64) -> D [64,192); odd: A [448,512) -> D [192,320) (fresh accumulators)
                    mma_f16_ts(tmem + (odd ? 192u : 64u), tmem + (odd ? 448u : 0u) + kk * 8,
                               sw128_desc(b_addr + (odd ? 32768u : 0u) + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                } else if (kCase == kSsDEachGroup) {
                    mma_f16_ss<1>(tmem + (odd ? 256u : 0u), sw128_desc(a_addr + off, 16, 1024),
                                  sw128_desc(b_addr + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                } else if (kCase == kTsAltMajor || kCase == kTsAltSameDesc) {
                    // TMEM: Q [0,64), S_a [64,192), S_b [192,320), O [320,448)
                    if (!odd) {
                        mma_f16_ts(tmem + 64u + 128u * which, tmem + kk * 8, sw128_desc(b_addr + off, 16, 1024),
                                   kIdS, kk > 0 ? 1u : 0u);
                    } else if (kCase == kTsAltMajor) {
                        mma_f16_ts(tmem + 320u, tmem + 64u + 128u * (which ^ 1u) + kk * 8,
                                   sw128_desc(b_addr + 32768 + kk * 2048, 16384, 1024), kIdO, 1u);
                    } else {
                        mma_f16_ts(tmem + 320u, tmem + 64u + 128u * (which ^ 1u) + kk * 8,
                                   sw128_desc(b_addr + 32768 + off, 16, 1024), kIdS, 1u);
                    }
                } else if (kCase == kSsAltMajor) {
                    if (!odd) {
                        mma_f16_ss<1>(tmem + 0u, sw128_desc(a_addr + off, 16, 1024), sw128_desc(b_addr + off, 16, 1024),
                                      kIdS, kk > 0 ? 1u : 0u);
                    } else {
                        mma_f16_ss<1>(tmem + 256u, sw128_desc(a_addr + off, 16, 1024),
                                      sw128_desc(b_addr + 32768 + kk * 2048, 16384, 1024), kIdO, 1u);
                    }
                } else if (kCase == kSsN256Reused || kCase == kSsN256Fresh) {
                    // B: 256 rows x 128 B per 64-deep K box (32 KiB), only box 0 is read
                    mma_f16_ss<1>(tmem + 256u * which, sw128_desc(a_addr + off, 16, 1024),
                                  sw128_desc(b_addr + b_tile + (kk & 3) * 32, 16, 1024), kIdW,
                                  kk > 0 ? 1u : 0u);
                } else if (pv) {
                    mma_f16_ts(tmem + 256u * which + 128u, tmem + 256u * (which ^ 1u) + kk * 8,
                               sw128_desc(b_addr + b_tile + kk * 2048, 16384, 1024), kIdO, 1u);
                } else {
                    mma_f16_ss<1>(tmem + 256u * which, sw128_desc(a_addr + off, 16, 1024),
                                  sw128_desc(b_addr + b_tile + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                }
            }
        }
        mma_commit(bar);
        bool done = false;
        for (long it = 0; it < 100000000L && !done; ++it) done = mbar_try_wait(bar, 0);
        cycles[kCase] = done ? clock64() - t0 : 0ull;
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc_fence_after();
        tmem_dealloc<1>(tmem, 512);
    }
}

template <int kCase>
bool run(unsigned long long* d) {
    if (cudaFuncSetAttribute(mma_rate<kCase>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
        cudaSuccess)
        return false;
    mma_rate<kCase><<<1, 128, kSmemBytes>>>(d);
    return cudaDeviceSynchronize() == cudaSuccess;
}

}  // namespace

int main() {
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, kCases * sizeof(unsigned long long)) != cudaSuccess) return 1;
    cudaMemset(d, 0, kCases * sizeof(unsigned long long));
    for (int rep = 0; rep < 2; ++rep) {
        if (!(run<kSsN128Reused>(d) && run<kSsN128Fresh>(d) && run<kTsN128Reused>(d) && run<kTsN128Fresh>(d) &&
              run<kSsN256Reused>(d) && run<kSsN256Fresh>(d) && run<kAttentionOrder>(d) && run<kTsAltMajor>(d) &&
              run<kTsAltSameDesc>(d) && run<kSsAltMajor>(d) && run<kTsAltNoHazard>(d) && run<kSsDEachGroup>(d) &&
              run<kTsAltMajorNoHazard>(d)))
            return 1;
    }
    unsigned long long h[kCases];
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    const char* names[kCases] = {"ss_n128_b_reused", "ss_n128_b_fresh", "ts_n128_b_reused", "ts_n128_b_fresh",
                                 "ss_n256_b_reused", "ss_n256_b_fresh", "attention_group_order",
                                 "ts_alternating_b_major", "ts_alternating_one_desc", "ss_alternating_b_major",
                                 "ts_alternating_no_tmem_overlap", "ss_accumulator_switch_each_group",
                                 "ts_alternating_b_major_no_overlap"};
    const int mma_cycles[kCases] = {64, 64, 64, 64, 128, 128, 64, 64, 64, 64, 64, 64, 64};  // at the dense f16 rate
    for (int c = 0; c < kCases; ++c)
        std::printf("{\"case\": \"%s\", \"cycles_per_mma\": %.1f, \"ideal\": %d}\n", names[c],
                    static_cast<double>(h[c]) / (kGroups * 8), mma_cycles[c]);
    return 0;
}
