// gemm.cuh — FP16 x FP16 -> FP32 row-major GEMM on sm_100a tensor cores.
//
// Replaces the SM7x WMMA/mma.sync kernel of ThunderKittens-SM7x
// (src/gemm.cu:87-166) behind the same contract (src/gemm.cu:184-206).
//
// Data layout: A is M x K row-major (K contiguous: a K-major MMA operand), B is
// K x N row-major (N contiguous: an MN-major operand), C is M x N row-major
// FP32. Both operands are fetched by TMA in 128-byte swizzled boxes:
//   A box  = 64 (K) x 128 (rows)        16 KiB, K-major SW128 canonical layout
//   B box  = 64 (N) x  64 (K rows)       8 KiB, MN-major SW128 canonical layout
// A stage holds one 64-deep K slice of the CTA's A rows and B columns. The ring
// of stages is filled by one producer warp and drained by one MMA warp whose
// elected lane issues tcgen05.mma (M = 128 per CTA, N = 256, K = 16) into a
// TMEM accumulator. Two 256-column accumulators (all 512 TMEM columns) let the
// four epilogue warps drain tile i (tcgen05.ld -> registers -> global) while
// the tensor core runs tile i + 1.
//
// kCtaGroup = 2 pairs two CTAs of a cluster on one 256 x 256 tile
// (tcgen05.mma.cta_group::2): each CTA loads its own 128 rows of A and its own
// 128 columns of B (no multicast), the even CTA issues the MMAs for both, and
// each CTA's TMEM receives its 128 rows of the 256 x 256 accumulator.
//
// The persistent grid walks output tiles in groups of Params::group_m tile-rows,
// column by column inside a group, so that the tiles resident at one time form a
// compact block that shares A row-blocks and B column-blocks in L2. C is written
// with evict-first stores so that the output stream does not displace A and B.
//
// Output shapes with too few tiles to fill the GPU split K: one work unit per
// (tile, K split). The splits of a tile either form a thread-block cluster and sum
// their partials over distributed shared memory (kEpiSplitCluster, one launch), or
// write partials that splitk_reduce_kernel sums; both in split order. Small such
// problems use 128-column tiles (kBN = 128: MMA N = 128, 256 TMEM columns).
#pragma once

#include "tk_ptx.cuh"
#include "tk_sm7x/tile_b200.cuh"

namespace tk {
namespace gemm {

constexpr int kBlockM = 128;   // rows of C per CTA
constexpr int kBlockN = 256;   // MMA N: columns of C per tile (128 in the small-M split-K variant)
constexpr int kBlockK = 64;    // K per pipeline stage (one 128-byte swizzle row)
constexpr int kMmaK = 16;      // K per tcgen05.mma (kind::f16)
constexpr int kGroupM = 16;    // default tile-rows per rasterisation group
constexpr int kThreads = 192;  // warps 0-3 epilogue, 4 producer, 5 MMA
constexpr int kMaxGatherRanks = 8;   // destinations of the all-gather epilogue

template <int kCtaGroup, int kBN = kBlockN>
struct Cfg {
    static constexpr int kTileM = kBlockM * kCtaGroup;        // rows per tile (per cluster)
    static constexpr int kBCols = kBN / kCtaGroup;            // B columns loaded per CTA
    static constexpr int kABytes = kBlockM * kBlockK * 2;     // 16 KiB
    static constexpr int kBBytes = kBlockK * kBCols * 2;      // 32 or 16 KiB
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = (kCtaGroup == 1 && kBN == 256) ? 4 : 6;
    static constexpr uint32_t kTmemCols = 2 * kBN;            // two FP32 accumulators
    // Row pitch (floats) of a partial tile in shared memory for kEpiSplitCluster: 16
    // bytes over a whole number of bank rows, so the 32 lanes' 16-byte stores of one
    // column quad fall on distinct banks eight lanes at a time.
    static constexpr int kRedStride = kBN + 4;
    static constexpr int kBarrierBytes = 256;
    // kEpiGather: a 32 x 33-float transpose buffer per epilogue warp, so that the
    // stores into the ranks' buffers are whole 128-byte row segments.
    static constexpr int kXposeBytes = 4 * 32 * 33 * 4;
    static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + kXposeBytes + 1024;  // + align slack
    static constexpr uint32_t kIdesc = idesc_f16_f32(kBlockM * kCtaGroup, kBN, 0, 1);
};

struct Params {
    int m, n, k;
    float* c;
    long long ldc;
    bool c_vec4;        // c 16-byte aligned and ldc % 4 == 0
    int m_tiles, n_tiles, k_blocks;
    int group_m;        // tile-rows per rasterisation group
    int num_tiles;      // m_tiles * n_tiles * k_splits work units
    // Split-K (small-M problems): unit t covers K blocks [ks * kb_per_split, ...)
    // and writes its partial C to ws[ks][m][n] (dense); splitk_reduce_kernel then
    // sums the splits in order into C (deterministic). k_splits == 1 writes C directly.
    int k_splits, kb_per_split;
    float* ws;
    // Fused row statistics: per-(row, n-tile) partials, then a finishing pass.
    float* partial;     // [m][n_tiles][2] (max, sum), or null
    // kEpiGather: row r of this GEMM goes to row dst_row0 + r of every dst[0..n_dst)
    // (this rank's gathered buffer and the peers' buffers mapped into this process),
    // leading dimension ldc, so the all-gather's transfer overlaps the MMAs tile by tile.
    float* dst[kMaxGatherRanks];
    int n_dst;
    long long dst_row0;
};

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int group_m, int* tm, int* tn) {
    const int per_group = group_m * n_tiles;
    const int group = t / per_group;
    const int first_m = group * group_m;
    const int rows = min(group_m, m_tiles - first_m);
    const int r = t - group * per_group;
    *tm = first_m + r % rows;
    *tn = r / rows;
}

// K-block of the i-th stage of a work unit: ascending for the CTA's even-numbered
// units and descending for its odd ones when K is not split. All CTAs turn round
// together, so a wave of tiles starts on the K-slices the previous wave read last,
// which are still in L2 (consecutive waves of one rasterisation group share their
// A rows). The order of the K-blocks changes the FP32 summation order of a tile,
// which stays inside the GEMM's error bound; split-K units keep ascending order, so
// both split reductions see identical partial sums.
#ifndef TK_GEMM_SNAKE_K
#define TK_GEMM_SNAKE_K 1
#endif
__device__ __forceinline__ int k_block_of(int i, int kb0, int kb1, int seq, const Params& p) {
    return (TK_GEMM_SNAKE_K != 0 && p.k_splits == 1 && (seq & 1)) ? kb1 - 1 - i : kb0 + i;
}

// Output tile and K-block range of work unit t.
__device__ __forceinline__ void work_coords(int t, const Params& p, int* tm, int* tn, int* kb0, int* kb1) {
    const int ks = t % p.k_splits;
    tile_coords(t / p.k_splits, p.m_tiles, p.n_tiles, p.group_m, tm, tn);
    *kb0 = ks * p.kb_per_split;
    *kb1 = min(*kb0 + p.kb_per_split, p.k_blocks);
}

using OpSumG = tk_sm7x::b200::op_sum;
using OpMaxG = tk_sm7x::b200::op_max;
using tk_sm7x::b200::tree16;  // canonical balanced tree over 16 consecutive values

// Level-by-level pairwise reduction of g[0..count) (count <= 16), odd last
// element carried up; fully unrolled so g stays in registers.
template <class Op>
__device__ __forceinline__ float pairwise16(float (&g)[16], int count) {
#pragma unroll
    for (int width = 16; width > 1; width >>= 1) {
#pragma unroll
        for (int i = 0; i < width / 2; ++i) {
            const bool has_low = 2 * i < count;
            const bool has_high = 2 * i + 1 < count;
            if (has_low) g[i] = has_high ? Op::apply(g[2 * i], g[2 * i + 1]) : g[2 * i];
        }
        count = (count + 1) >> 1;
    }
    return g[0];
}

// Epilogue statistics per (row, 256-column tile), written to Params::partial:
enum Stats : int {
    kStatsNone = 0,
    kStatsMaxSum = 1,   // (row max, row sum) of the tile's columns, fixed pairwise order
    kStatsSoftmax = 2,  // (row max m_t, sum of exp(c - m_t)) for a full-row softmax
    kEpiGather = 3,     // no statistics; each row stored to every Params::dst (multi-GPU all-gather)
    // Split-K reduced inside the cluster: the k_splits CTAs of one output tile form a
    // cluster (CTA rank = split index, one work unit per CTA). Each leaves its partial
    // tile in its own shared memory; after a cluster barrier every CTA sums its share
    // of the tile over all splits in split order (distributed shared memory) into C.
    kEpiSplitCluster = 4,
};

template <int kCtaGroup, int kStats, int kBN = kBlockN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const Params p) {
    using C = Cfg<kCtaGroup, kBN>;
    static_assert(kBN == kBlockN || ((kStats == kStatsNone || kStats == kEpiSplitCluster) && kCtaGroup == 1),
                  "128-column tiles only for plain single-CTA tiles");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);

    const uint32_t barriers = base + C::kStages * C::kStageBytes;
    auto full_bar = [&](int s) { return barriers + 8u * s; };
    auto empty_bar = [&](int s) { return barriers + 8u * (C::kStages + s); };
    auto tfull_bar = [&](int b) { return barriers + 8u * (2 * C::kStages + b); };
    auto tempty_bar = [&](int b) { return barriers + 8u * (2 * C::kStages + 2 + b); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kStages * C::kStageBytes + 8 * (2 * C::kStages + 4));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_id();
    const uint32_t lane = lane_id();
    const uint32_t rank = kCtaGroup == 2 ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int cluster_id = static_cast<int>(blockIdx.x) / kCtaGroup;
    const int num_clusters = static_cast<int>(gridDim.x) / kCtaGroup;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 4 * kCtaGroup);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 4 && lane == 0) {
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
    }
    if (warp == 5) {
        tmem_alloc<kCtaGroup>(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish<kCtaGroup>();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kCtaGroup == 2) cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // A programmatic dependent (the split-K reduction) may be scheduled now; it
    // waits for this grid's completion before reading anything.
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 4) {
        // ---------------- producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0;
        bool ok = true;
        const uint32_t leader_full0 = kCtaGroup == 2 ? mapa_shared(full_bar(0), 0) : full_bar(0);
        for (int t = cluster_id, seq = 0; t < p.num_tiles && ok; t += num_clusters, ++seq) {
            int tm, tn, kb0, kb1;
            work_coords(t, p, &tm, &tn, &kb0, &kb1);
            const int row0 = tm * C::kTileM + static_cast<int>(rank) * kBlockM;
            const int col0 = tn * kBN + static_cast<int>(rank) * C::kBCols;
            for (int i = 0; i < kb1 - kb0; ++i) {
                const int kb = k_block_of(i, kb0, kb1, seq, p);
                if (!mbar_wait_warp(empty_bar(stage), phase ^ 1u, kFaultProducerWait, abort_flag)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t a_dst = base + stage * C::kStageBytes;
                    const uint32_t b_dst = a_dst + C::kABytes;
                    if constexpr (kCtaGroup == 1) {
                        mbar_arrive_expect_tx(full_bar(stage), C::kStageBytes);
                        tma_load_2d(a_dst, &map_a, full_bar(stage), kb * kBlockK, row0);
#pragma unroll
                        for (int j = 0; j < C::kBCols / 64; ++j)
                            tma_load_2d(b_dst + j * 8192, &map_b, full_bar(stage), col0 + j * 64,
                                        kb * kBlockK);
                    } else {
                        if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * C::kStageBytes);
                        const uint32_t fb = leader_full0 + 8u * stage;
                        tma_load_2d_pair(a_dst, &map_a, fb, kb * kBlockK, row0);
#pragma unroll
                        for (int j = 0; j < C::kBCols / 64; ++j)
                            tma_load_2d_pair(b_dst + j * 8192, &map_b, fb, col0 + j * 64,
                                             kb * kBlockK);
                    }
                }
                __syncwarp();
                ++issued;
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        // Drain: the last loads issued by this CTA must land before it may exit.
        if (!ok && leader) {
            int s = stage;
            uint32_t ph = phase;
            for (int i = 0; i < min(issued, C::kStages); ++i) {
                if (--s < 0) {
                    s = C::kStages - 1;
                    ph ^= 1u;
                }
                mbar_wait_warp(full_bar(s), ph, kFaultDrainWait, nullptr);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer (leader CTA) ----------------
        if (leader) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = cluster_id; t < p.num_tiles && ok; t += num_clusters) {
                if (!mbar_wait_warp(tempty_bar(acc), acc_phase ^ 1u, kFaultMmaWait, abort_flag)) break;
                tc_fence_after();
                int tm, tn, kb0, kb1;
                work_coords(t, p, &tm, &tn, &kb0, &kb1);
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
                for (int kb = kb0; kb < kb1; ++kb) {  // stages arrive in the producer's K order
                    if (!mbar_wait_warp(full_bar(stage), phase, kFaultMmaWait, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t a_addr = base + stage * C::kStageBytes;
                        const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
                        for (int kk = 0; kk < kBlockK / kMmaK; ++kk) {
                            const uint64_t a_desc = sw128_desc(a_addr + kk * 32, 16, 1024);
                            const uint64_t b_desc = sw128_desc(b_addr + kk * 2048, 8192, 1024);
                            mma_f16_ss<kCtaGroup>(d_tmem, a_desc, b_desc, C::kIdesc,
                                                  (kb > kb0 || kk > 0) ? 1u : 0u);
                        }
                        if constexpr (kCtaGroup == 1) {
                            mma_commit(empty_bar(stage));
                        } else {
                            mma_commit_pair(empty_bar(stage), 0x3);
                        }
                    }
                    __syncwarp();
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (lane == 0) {
                    if constexpr (kCtaGroup == 1) {
                        mma_commit(tfull_bar(acc));
                    } else {
                        mma_commit_pair(tfull_bar(acc), 0x3);
                    }
                }
                __syncwarp();
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue warps 0-3: TMEM -> registers -> global ----------------
        int acc = 0;
        uint32_t acc_phase = 0;
        const uint32_t tempty_remote =
            kCtaGroup == 2 ? mapa_shared(tempty_bar(0), 0) : tempty_bar(0);
        for (int t = cluster_id; t < p.num_tiles; t += num_clusters) {
            int tm, tn, kb0, kb1;
            work_coords(t, p, &tm, &tn, &kb0, &kb1);
            if (!mbar_wait_warp(tfull_bar(acc), acc_phase, kFaultEpilogueWait, abort_flag)) break;
            tc_fence_after();
            const long long row =
                static_cast<long long>(tm) * C::kTileM + rank * kBlockM + warp * 32 + lane;
            const int col_base = tn * kBN;
            const bool row_ok = row < p.m;
            const bool split = kStats != kEpiSplitCluster && p.k_splits > 1;
            float* crow = split ? p.ws + (static_cast<long long>(t % p.k_splits) * p.m + row) * p.n
                                : p.c + row * p.ldc;
            const bool vec4 = split || p.c_vec4;
            const uint32_t t_addr = tmem_base + ((warp * 32u) << 16) + static_cast<uint32_t>(acc * kBN);
            float gmax[16], gsum[16];
#pragma unroll
            for (int chunk = 0; chunk < kBN / 32; ++chunk) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_addr + chunk * 32, r);
                tmem_wait_ld();
                const int col0 = col_base + chunk * 32;
                if constexpr (kStats == kEpiGather) {
                    // Through shared memory: lane l holds row (32 warp + l) of the chunk;
                    // after the transpose, one store instruction writes one row's 32
                    // consecutive columns (128 bytes) into every destination.
                    float* xp = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes + C::kBarrierBytes) +
                                warp * (32 * 33);
#pragma unroll
                    for (int q = 0; q < 32; ++q) xp[lane * 33 + q] = __uint_as_float(r[q]);
                    __syncwarp();
                    const long long row_first = static_cast<long long>(tm) * C::kTileM + rank * kBlockM + warp * 32;
                    const bool col_ok = col0 + static_cast<int>(lane) < p.n;
                    for (int i = 0; i < 32; ++i) {
                        const long long rr = row_first + i;
                        if (rr >= p.m) break;  // warp-uniform
                        const float v = xp[i * 33 + lane];
                        if (col_ok) {
#pragma unroll
                            for (int d = 0; d < kMaxGatherRanks; ++d) {
                                if (d >= p.n_dst) break;
                                p.dst[d][(p.dst_row0 + rr) * p.ldc + col0 + lane] = v;
                            }
                        }
                    }
                    __syncwarp();
                }
                if constexpr (kStats == kEpiSplitCluster) {
                    // Partial rows stay in this CTA's shared memory (the pipeline stages
                    // are idle: every load of the CTA's one work unit has been consumed).
                    if (row_ok) {
                        float* prow = reinterpret_cast<float*>(smem) + (warp * 32 + lane) * C::kRedStride + chunk * 32;
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            *reinterpret_cast<float4*>(prow + 4 * q) =
                                make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                            __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
                    }
                }
                constexpr int kDsts = (kStats == kEpiGather || kStats == kEpiSplitCluster) ? 0 : 1;
#pragma unroll
                for (int d = 0; d < kDsts; ++d) {
                    float* const drow = crow;
                    if (row_ok) {
                        if (vec4) {
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                if (col0 + q * 4 < p.n) {
                                    float4 v = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                           __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
                                    __stcs(reinterpret_cast<float4*>(drow + col0 + q * 4), v);
                                }
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 32; ++q)
                                if (col0 + q < p.n) __stcs(drow + col0 + q, __uint_as_float(r[q]));
                        }
                    }
                }
                if constexpr (kStats == kStatsMaxSum || kStats == kStatsSoftmax) {
                    float x[32];
#pragma unroll
                    for (int q = 0; q < 32; ++q) x[q] = __uint_as_float(r[q]);
                    gmax[2 * chunk] = tree16<OpMaxG>(x);
                    gmax[2 * chunk + 1] = tree16<OpMaxG>(x + 16);
                    if constexpr (kStats == kStatsMaxSum) {
                        gsum[2 * chunk] = tree16<OpSumG>(x);
                        gsum[2 * chunk + 1] = tree16<OpSumG>(x + 16);
                    }
                }
            }
            if constexpr (kStats == kStatsSoftmax) {
                // Second read of the accumulator: sum of exp(c - m_t) over this
                // tile's valid columns, m_t the tile-row max (warp-uniform loop).
                const int groups = max(0, min(16, (p.n - col_base) / 16));
                const float m_t = pairwise16<OpMaxG>(gmax, groups);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int chunk = 0; chunk < kBN / 32; ++chunk) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_addr + chunk * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 32; ++q) {
                        if (col_base + chunk * 32 + q < p.n)
                            acc[q & 3] += tk_sm7x::b200::ex2_approx(
                                (__uint_as_float(r[q]) - m_t) * 1.4426950408889634f);
                    }
                }
                gmax[0] = m_t;
                gsum[0] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (kCtaGroup == 1) {
                    mbar_arrive(tempty_bar(acc));
                } else {
                    mbar_arrive_cluster(tempty_remote + 8u * acc);
                }
            }
            if constexpr (kStats == kStatsMaxSum) {
                if (row_ok) {
                    const int groups = min(16, (p.n - col_base) / 16);
                    const float mx = pairwise16<OpMaxG>(gmax, groups);
                    const float sm = pairwise16<OpSumG>(gsum, groups);
                    float2* dst = reinterpret_cast<float2*>(p.partial) + (row * p.n_tiles + tn);
                    *dst = make_float2(mx, sm);
                }
            }
            if constexpr (kStats == kStatsSoftmax) {
                if (row_ok) {
                    float2* dst = reinterpret_cast<float2*>(p.partial) + (row * p.n_tiles + tn);
                    *dst = make_float2(gmax[0], gsum[0]);
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (kCtaGroup == 2) cluster_sync();
    if constexpr (kStats == kEpiSplitCluster) {
        static_assert(kCtaGroup == 1, "the in-cluster split-K reduction runs on single-CTA tiles");
        static_assert(kBlockM * C::kRedStride * 4 <= C::kStages * C::kStageBytes,
                      "partial tile larger than the pipeline stages");
        // Every CTA reaches both barriers, also after a timed-out wait (its partial is
        // then not used: the fault is recorded and the call reports it).
        cluster_sync();  // every split's partial is in its CTA's shared memory
        int tm, tn, kb0, kb1;
        work_coords(static_cast<int>(blockIdx.x), p, &tm, &tn, &kb0, &kb1);
        const int rows = min(kBlockM, p.m - tm * kBlockM);
        const int quads_per_row = min(kBN, p.n - tn * kBN) / 4;
        const int quads = rows * quads_per_row;
        const int my = static_cast<int>(cluster_ctarank());
        const int q_end = quads * (my + 1) / p.k_splits;
        for (int q = quads * my / p.k_splits + static_cast<int>(threadIdx.x); q < q_end; q += kThreads) {
            const int r = q / quads_per_row;
            const int c4 = (q - r * quads_per_row) * 4;
            const uint32_t local = base + static_cast<uint32_t>((r * C::kRedStride + c4) * 4);
            // Split order, as splitk_reduce_kernel: bit-identical results.
            float4 acc = ld_shared_cluster_f4(mapa_shared(local, 0));
            for (int sp = 1; sp < p.k_splits; ++sp) {
                const float4 v = ld_shared_cluster_f4(mapa_shared(local, static_cast<uint32_t>(sp)));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            float* dst = p.c + (static_cast<long long>(tm) * kBlockM + r) * p.ldc + tn * kBN + c4;
            if (p.c_vec4) {
                *reinterpret_cast<float4*>(dst) = acc;
            } else {
                dst[0] = acc.x;
                dst[1] = acc.y;
                dst[2] = acc.z;
                dst[3] = acc.w;
            }
        }
        cluster_sync();  // no CTA leaves while another still reads its shared memory
    }
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc<kCtaGroup>(tmem_base, C::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Small-M GEMM (M <= 64, decode-shaped): C^T = B^T A^T on the tensor core, so the
// few rows of A become the MMA's N (16..64) and 128 columns of B its M. A tile of
// 128 output columns then costs 4 MMAs of 128 x m_pad x 16 per 64-deep K block
// (8x less tensor work than 128-row tiles of which M rows are used), and the kernel
// streams B, the only large operand, at the rate of the loads in flight.
//   MMA A = B tile (64 N x 64 K TMA boxes, MN-major: the same boxes as the GEMM's B)
//   MMA B = A rows (64 K x m_pad rows, K-major)
//   D (TMEM) = 128 lanes (output columns) x m_pad columns (output rows)
// One CTA per (128-column tile, K split); small enough for two CTAs per SM. The K
// splits of a tile form a cluster (CTA rank = split) and sum their partials in split
// order over distributed shared memory (kCluster), or write them to scratch for
// splitk_reduce_kernel (same order, same bits).
// ---------------------------------------------------------------------------
constexpr int kSkinnyStages = 4;
constexpr int kSkinnyBN = 128;
constexpr int kSkinnyMaxM = 64;
constexpr int kSkinnyStageBytes = 2 * 8192 + kSkinnyMaxM * 128;  // B boxes + A box (up to 64 rows)
constexpr int kSkinnySmemBytes = kSkinnyStages * kSkinnyStageBytes + 256 + 1024;

struct SkinnyParams {
    int m, n, k, m_pad;
    float* c;
    long long ldc;
    bool c_vec4;
    int n_tiles, k_blocks, k_splits, kb_per_split;
    float* ws;  // split partials [k_splits][m][n] (second-kernel form), or null
};

template <bool kCluster>
__global__ void __launch_bounds__(kThreads, 2)
    skinny_kernel(const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_a,
                  const SkinnyParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);
    const uint32_t bars = base + kSkinnyStages * kSkinnyStageBytes;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (kSkinnyStages + s); };
    const uint32_t tfull = bars + 8u * (2 * kSkinnyStages);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSkinnyStages * kSkinnyStageBytes + 8 * (2 * kSkinnyStages + 1));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_id();
    const uint32_t lane = lane_id();
    const int unit = static_cast<int>(blockIdx.x);
    const int split = unit % p.k_splits;
    const int tile = unit / p.k_splits;
    const int n0 = tile * kSkinnyBN;
    const int kb0 = split * p.kb_per_split;
    const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
    const uint32_t tmem_cols = p.m_pad <= 32 ? 32u : 64u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSkinnyStages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(tfull, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 4 && lane == 0) {
        tma_prefetch_desc(&map_b);
        tma_prefetch_desc(&map_a);
    }
    if (warp == 5) {
        tmem_alloc<1>(smem_u32(tmem_slot), tmem_cols);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    const uint32_t a_bytes = static_cast<uint32_t>(p.m_pad) * 128u;
    if (warp == 4) {
        // ---------------- producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait_warp(empty_bar(stage), phase ^ 1u, kFaultProducerWait, abort_flag)) {
                ok = false;
                break;
            }
            if (lane == 0) {
                const uint32_t dst = base + stage * kSkinnyStageBytes;
                mbar_arrive_expect_tx(full_bar(stage), 2u * 8192u + a_bytes);
                tma_load_2d(dst, &map_b, full_bar(stage), n0, kb * kBlockK);
                tma_load_2d(dst + 8192, &map_b, full_bar(stage), n0 + 64, kb * kBlockK);
                tma_load_2d(dst + 16384, &map_a, full_bar(stage), kb * kBlockK, 0);
            }
            __syncwarp();
            ++issued;
            if (++stage == kSkinnyStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (!ok) {
            int s = stage;
            uint32_t ph = phase;
            for (int i = 0; i < min(issued, kSkinnyStages); ++i) {
                if (--s < 0) {
                    s = kSkinnyStages - 1;
                    ph ^= 1u;
                }
                mbar_wait_warp(full_bar(s), ph, kFaultDrainWait, nullptr);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        const uint32_t idesc = idesc_f16_f32(kSkinnyBN, p.m_pad, 1, 0);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait_warp(full_bar(stage), phase, kFaultMmaWait, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (lane == 0) {
                const uint32_t b_tile = base + stage * kSkinnyStageBytes;
                const uint32_t a_rows = b_tile + 16384;
#pragma unroll
                for (int kk = 0; kk < kBlockK / kMmaK; ++kk)
                    mma_f16_ss<1>(tmem, sw128_desc(b_tile + kk * 2048, 8192, 1024), sw128_desc(a_rows + kk * 32, 16, 1024),
                                  idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                mma_commit(empty_bar(stage));
            }
            __syncwarp();
            if (++stage == kSkinnyStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (ok && lane == 0) mma_commit(tfull);
        __syncwarp();
    } else {
        // ---------------- epilogue warps 0-3: lane = output column ----------------
        const bool have = kb1 > kb0;
        const bool ok = !have || mbar_wait_warp(tfull, 0u, kFaultEpilogueWait, abort_flag);
        tc_fence_after();
        const int col = n0 + static_cast<int>(warp * 32 + lane);
        const bool col_ok = col < p.n;
        float* part = reinterpret_cast<float*>(smem);  // [m_pad][128], over the consumed stages
        for (int c = 0; c < p.m_pad / 16; ++c) {
            uint32_t r[16];
            if (have && ok) {
                tmem_ld_32x32b_x16(tmem + ((warp * 32u) << 16) + 16u * c, r);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) r[i] = 0u;  // an empty K range contributes zero
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int row = 16 * c + i;
                const float v = __uint_as_float(r[i]);
                if constexpr (kCluster) {
                    part[row * kSkinnyBN + warp * 32 + lane] = v;
                } else if (row < p.m && col_ok) {
                    if (p.ws != nullptr)
                        p.ws[(static_cast<long long>(split) * p.m + row) * p.n + col] = v;
                    else
                        __stcs(p.c + row * p.ldc + col, v);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (kCluster) {
        // Every CTA of the cluster reaches both barriers, also after a timed-out wait
        // (the fault is recorded and the call reports it).
        cluster_sync();  // every split's partial is in its CTA's shared memory
        const int quads = p.m * (kSkinnyBN / 4);
        const int my = static_cast<int>(cluster_ctarank());
        const int q_end = quads * (my + 1) / p.k_splits;
        for (int q = quads * my / p.k_splits + static_cast<int>(threadIdx.x); q < q_end; q += kThreads) {
            const int row = q / (kSkinnyBN / 4);
            const int c4 = (q - row * (kSkinnyBN / 4)) * 4;
            if (n0 + c4 >= p.n) continue;  // n is a multiple of 16: a quad is all in or all out
            const uint32_t local = base + static_cast<uint32_t>((row * kSkinnyBN + c4) * 4);
            // Split order, as splitk_reduce_kernel: bit-identical results.
            float4 acc = ld_shared_cluster_f4(mapa_shared(local, 0));
            for (int sp = 1; sp < p.k_splits; ++sp) {
                const float4 v = ld_shared_cluster_f4(mapa_shared(local, static_cast<uint32_t>(sp)));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            float* dst = p.c + static_cast<long long>(row) * p.ldc + n0 + c4;
            if (p.c_vec4) {
                __stcs(reinterpret_cast<float4*>(dst), acc);
            } else {
                dst[0] = acc.x;
                dst[1] = acc.y;
                dst[2] = acc.z;
                dst[3] = acc.w;
            }
        }
        cluster_sync();  // no CTA leaves while another still reads its shared memory
    }
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc<1>(tmem, tmem_cols);
    }
}

// Finishing pass of the fused row statistics: per row, combine the per-tile
// partials in tile order with the same pairwise rule (binary-counter form: a
// stack of complete power-of-two blocks, merged right to left at the end, which
// equals the level-by-level pairing with the odd element carried up).
//
// A GEMM that gave up on a bounded wait leaves some partials unwritten; while the
// status word records such a fault the pass writes NaN instead of combining them.
__global__ void rowstats_finish_kernel(const float2* partial, int m, int n_tiles, float* row_max,
                                       float* row_sum) {
    const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (row >= m) return;
    if (*static_cast<volatile unsigned int*>(&g_tk_status) != 0u) {
        row_max[row] = __int_as_float(0x7fc00000);
        row_sum[row] = __int_as_float(0x7fc00000);
        return;
    }
    float smax[32], ssum[32];
    int ssize[32];
    int top = 0;
    const float2* src = partial + row * n_tiles;
    for (int i = 0; i < n_tiles; ++i) {
        float2 v = src[i];
        float vmax = v.x, vsum = v.y;
        int size = 1;
        while (top > 0 && ssize[top - 1] == size) {
            --top;
            vmax = OpMaxG::apply(smax[top], vmax);
            vsum = OpSumG::apply(ssum[top], vsum);
            size *= 2;
        }
        smax[top] = vmax;
        ssum[top] = vsum;
        ssize[top] = size;
        ++top;
    }
    float vmax = smax[top - 1], vsum = ssum[top - 1];
    for (int i = top - 2; i >= 0; --i) {
        vmax = OpMaxG::apply(smax[i], vmax);
        vsum = OpSumG::apply(ssum[i], vsum);
    }
    row_max[row] = vmax;
    row_sum[row] = vsum;
}

// Full-row softmax from the per-tile (m_t, sum exp(c - m_t)) pairs, one warp per
// row: the lanes merge the pairs (row max M, normaliser S = sum s_t exp(m_t - M),
// a fixed shuffle order, so the result is deterministic), then the warp writes
// p = exp(c - M) / S over the row. p may be c itself: each element is read before
// the same lane overwrites it. While the status word records a fault (a GEMM that
// gave up on a wait, leaving pairs unwritten) every p is NaN.
__global__ void __launch_bounds__(256) rowsoftmax_apply_kernel(const float2* partial, int m, int n,
                                                               int n_tiles, const float* c, long long ldc,
                                                               float* p, long long ldp, bool vec4) {
    constexpr float kLog2e = 1.4426950408889634f;
    const bool faulted = *static_cast<volatile unsigned int*>(&g_tk_status) != 0u;
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    for (long long row = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); row < m;
         row += warps) {
        const float2* src = partial + row * n_tiles;
        float big = -INFINITY;
        for (int t = lane; t < n_tiles; t += 32) big = fmaxf(big, src[t].x);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) big = fmaxf(big, __shfl_xor_sync(0xffffffffu, big, o));
        float total = 0.0f;
        for (int t = lane; t < n_tiles; t += 32)
            total += src[t].y * tk_sm7x::b200::ex2_approx((src[t].x - big) * kLog2e);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
        const float inv = faulted ? __int_as_float(0x7fc00000) : __frcp_rn(total);
        const float* crow = c + row * ldc;
        float* prow = p + row * ldp;
        if (vec4) {
            for (int j = lane * 4; j < n; j += 128) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>(crow + j));
                float4 o;
                o.x = tk_sm7x::b200::ex2_approx((v.x - big) * kLog2e) * inv;
                o.y = tk_sm7x::b200::ex2_approx((v.y - big) * kLog2e) * inv;
                o.z = tk_sm7x::b200::ex2_approx((v.z - big) * kLog2e) * inv;
                o.w = tk_sm7x::b200::ex2_approx((v.w - big) * kLog2e) * inv;
                __stcs(reinterpret_cast<float4*>(prow + j), o);
            }
        } else {
            for (int j = lane; j < n; j += 32)
                prow[j] = tk_sm7x::b200::ex2_approx((crow[j] - big) * kLog2e) * inv;
        }
    }
}

// Sums the split-K partials ws[0..splits)[m][n] in split order into C (ldc).
// Launched as a programmatic dependent of the GEMM: it may start while the GEMM's
// last CTAs finish, and griddepcontrol.wait holds it until the GEMM has completed
// and its partials are visible.
__global__ void splitk_reduce_kernel(const float* ws, int splits, int m, int n, float* c, long long ldc,
                                     bool c_vec4) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const long long quads = static_cast<long long>(m) * (n / 4);
    const long long plane = static_cast<long long>(m) * n;
    for (long long q = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; q < quads;
         q += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long row = q / (n / 4);
        const int col = static_cast<int>(q - row * (n / 4)) * 4;
        const float* src = ws + row * n + col;
        float4 acc = *reinterpret_cast<const float4*>(src);
        for (int s = 1; s < splits; ++s) {
            const float4 v = *reinterpret_cast<const float4*>(src + s * plane);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        float* dst = c + row * ldc + col;
        if (c_vec4) {
            *reinterpret_cast<float4*>(dst) = acc;
        } else {
            dst[0] = acc.x;
            dst[1] = acc.y;
            dst[2] = acc.z;
            dst[3] = acc.w;
        }
    }
}

// Copies a binary16 matrix with an arbitrary leading dimension / alignment into
// a dense 16-byte-aligned buffer (rows x cols, leading dimension cols) so that
// TMA can read it. Used only when the caller's operand cannot be described by a
// tensor map (row pitch not a multiple of 16 bytes or a misaligned base).
__global__ void repack_f16_kernel(const uint16_t* src, long long ld, uint16_t* dst, long long rows,
                                  int cols) {
    const long long total = rows * cols;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / cols;
        const long long c = i - r * cols;
        dst[i] = src[r * ld + c];
    }
}

}  // namespace gemm
}  // namespace tk
