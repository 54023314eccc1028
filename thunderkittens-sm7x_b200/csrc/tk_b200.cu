// tk_b200.cu — the library's single translation unit and its C ABI
// (include/tk_b200.h). Argument validation and error-state rules follow
// ThunderKittens-SM7x src/gemm.cu:184-206 and src/attention.cu:62-86:
// invalid arguments return cudaErrorInvalidValue before anything else happens
// (no launch, outputs untouched, the pending CUDA error left in place); a valid
// call clears the pending error, enqueues, and returns cudaGetLastError().

#include "tk_b200.h"

#include <atomic>
#include <climits>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "attention.cuh"
#include "attention_pair.cuh"
#include "gemm.cuh"
#include "rowops.cuh"
#include "tk_host.cuh"

namespace {

using tk::host::current_device;

constexpr int kAbiVersion = 101;

// ---------------------------------------------------------------------------
// Tile row operations
// ---------------------------------------------------------------------------

template <int kOps, bool kVec>
void launch_rowops_typed(const float* tiles, size_t n_tiles, float* s, float* m, float* sm, float* cs,
                         int sm_count, cudaStream_t stream) {
    // Resident blocks per SM, looked up once (several host threads may race to do
    // it; each stores the same value).
    static std::atomic<int> cached_blocks_per_sm{0};
    int blocks_per_sm = cached_blocks_per_sm.load(std::memory_order_acquire);
    if (blocks_per_sm == 0) {
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &occ, tk::rowops::tile_row_ops_kernel<kOps, kVec>, tk::rowops::kThreads, 0) !=
                cudaSuccess ||
            occ <= 0) {
            static_cast<void>(cudaGetLastError());
            occ = 4;
        }
        blocks_per_sm = occ;
        cached_blocks_per_sm.store(occ, std::memory_order_release);
    }
    const size_t tiles_per_block = (tk::rowops::kThreads / 32) * tk::rowops::kTilesPerWarpStep;
    const size_t needed = (n_tiles + tiles_per_block - 1) / tiles_per_block;
    const size_t cap = static_cast<size_t>(sm_count) * blocks_per_sm;
    const unsigned grid = static_cast<unsigned>(needed < cap ? needed : cap);
    tk::rowops::tile_row_ops_kernel<kOps, kVec>
        <<<grid, tk::rowops::kThreads, 0, stream>>>(tiles, n_tiles, s, m, sm, cs);
}

template <int kOps>
void launch_rowops_ops(bool vec, const float* tiles, size_t n_tiles, float* s, float* m, float* sm,
                       float* cs, int sm_count, cudaStream_t stream) {
    if (vec) {
        launch_rowops_typed<kOps, true>(tiles, n_tiles, s, m, sm, cs, sm_count, stream);
    } else {
        launch_rowops_typed<kOps, false>(tiles, n_tiles, s, m, sm, cs, sm_count, stream);
    }
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

cudaError_t rowops(const float* tiles, size_t n_tiles, float* sum_out, float* max_out,
                   float* softmax_out, float* causal_out, bool allow_inplace, cudaStream_t stream) {
    if (tiles == nullptr || (sum_out == nullptr && max_out == nullptr && softmax_out == nullptr &&
                             causal_out == nullptr)) {
        return cudaErrorInvalidValue;
    }
    if (n_tiles > SIZE_MAX / 1024) return cudaErrorInvalidValue;
    const float* outs[4] = {sum_out, max_out, softmax_out, causal_out};
    const size_t out_bytes[4] = {n_tiles * 64, n_tiles * 64, n_tiles * 1024, n_tiles * 1024};
    const size_t in_bytes = n_tiles * 1024;
    for (int i = 0; i < 4; ++i) {
        if (outs[i] == nullptr) continue;
        if (!aligned(outs[i], 4)) return cudaErrorInvalidValue;
        if (tk::host::ranges_overlap(outs[i], out_bytes[i], tiles, in_bytes) &&
            !(allow_inplace && static_cast<const void*>(outs[i]) == static_cast<const void*>(tiles) &&
              out_bytes[i] == in_bytes)) {
            return cudaErrorInvalidValue;
        }
        for (int j = i + 1; j < 4; ++j) {
            if (outs[j] != nullptr && tk::host::ranges_overlap(outs[i], out_bytes[i], outs[j], out_bytes[j]))
                return cudaErrorInvalidValue;
        }
    }
    if (!aligned(tiles, 4)) return cudaErrorInvalidValue;
    int sm_count = 0;
    cudaError_t err = current_device(nullptr, &sm_count);
    if (err != cudaSuccess) return err;
    static_cast<void>(cudaGetLastError());
    if (n_tiles == 0) return cudaSuccess;
    bool vec = aligned(tiles, 16);
    for (int i = 0; i < 4; ++i)
        if (outs[i] != nullptr) vec = vec && aligned(outs[i], 16);
    const int ops = (sum_out ? tk::rowops::kSum : 0) | (max_out ? tk::rowops::kMax : 0) |
                    (softmax_out ? tk::rowops::kSoftmax : 0) | (causal_out ? tk::rowops::kCausal : 0);
    switch (ops) {
#define TK_ROWOPS_CASE(N)                                                                              \
    case N:                                                                                            \
        launch_rowops_ops<N>(vec, tiles, n_tiles, sum_out, max_out, softmax_out, causal_out, sm_count, \
                             stream);                                                                  \
        break;
        TK_ROWOPS_CASE(1) TK_ROWOPS_CASE(2) TK_ROWOPS_CASE(3) TK_ROWOPS_CASE(4) TK_ROWOPS_CASE(5)
        TK_ROWOPS_CASE(6) TK_ROWOPS_CASE(7) TK_ROWOPS_CASE(8) TK_ROWOPS_CASE(9) TK_ROWOPS_CASE(10)
        TK_ROWOPS_CASE(11) TK_ROWOPS_CASE(12) TK_ROWOPS_CASE(13) TK_ROWOPS_CASE(14) TK_ROWOPS_CASE(15)
#undef TK_ROWOPS_CASE
        default: break;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------

// Process-wide tuning knobs, read by every call (possibly from several host threads).
std::atomic<int> g_gemm_cta_group_override{0};  // 0 = choose by problem size

template <int kCtaGroup, int kStats, int kBN = tk::gemm::kBlockN>
cudaError_t launch_gemm_kernel(const CUtensorMap& ma, const CUtensorMap& mb, const tk::gemm::Params& p,
                               int device, int sm_count, cudaStream_t stream) {
    using Cfg = tk::gemm::Cfg<kCtaGroup, kBN>;
    auto kernel = tk::gemm::gemm_kernel<kCtaGroup, kStats, kBN>;
    // Per-device shared-memory opt-in, done once; concurrent first calls may both
    // set the (idempotent) attribute.
    static std::atomic<bool> configured[tk::host::kMaxDevices];
    if (!configured[device].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured[device].store(true, std::memory_order_release);
    }
    const int max_clusters = sm_count / kCtaGroup;
    const int clusters = p.num_tiles < max_clusters ? p.num_tiles : max_clusters;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * kCtaGroup));
    cfg.blockDim = dim3(tk::gemm::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCtaGroup;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, ma, mb, p);
}

// Split-K with the reduction inside the kernel: grid = every work unit, clusters
// of k_splits CTAs (one output tile each).
template <int kBN>
cudaError_t launch_gemm_split_cluster(const CUtensorMap& ma, const CUtensorMap& mb, const tk::gemm::Params& p,
                                      cudaStream_t stream) {
    using Cfg = tk::gemm::Cfg<1, kBN>;
    auto kernel = tk::gemm::gemm_kernel<1, tk::gemm::kEpiSplitCluster, kBN>;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(p.num_tiles));
    cfg.blockDim = dim3(tk::gemm::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(p.k_splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, ma, mb, p);
}

// How many clusters of `splits` CTAs of the in-cluster split-K kernel with
// kBN-column tiles can be resident at once on `device` (cached; 0 when the query
// fails). Also sets the kernel's shared-memory limit, which its launch needs.
template <int kBN>
int split_cluster_capacity(int device, int splits) {
    static std::atomic<int> cache[tk::host::kMaxDevices][9];
    static std::atomic<bool> configured[tk::host::kMaxDevices];
    int v = cache[device][splits].load(std::memory_order_acquire);
    if (v != 0) return v < 0 ? 0 : v;
    using Cfg = tk::gemm::Cfg<1, kBN>;
    auto kernel = tk::gemm::gemm_kernel<1, tk::gemm::kEpiSplitCluster, kBN>;
    if (!configured[device].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) !=
            cudaSuccess) {
            static_cast<void>(cudaGetLastError());
            return 0;
        }
        configured[device].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(splits));
    cfg.blockDim = dim3(tk::gemm::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
        static_cast<void>(cudaGetLastError());
        clusters = 0;
    }
    cache[device][splits].store(clusters > 0 ? clusters : -1, std::memory_order_release);
    return clusters;
}

// Tile-rows per rasterisation group. The tiles in flight at one time (one per CTA or
// CTA pair: 148 or 74 on B200) walk a group column by column. Measured on B200
// (CTA-pair tiles, TFLOP/s for 4 / 6 / 8 / 12 / 16 / 32 rows): 8192^3 1323 / 1360 /
// 1389 / 1387 / 1423 / 1215; 16384 x 4096 x 14336 (16 tile-columns) 1216 / 1214 /
// 1063 / 1070 / 1073 / 1202. DRAM reads at 8192^3 stay 4.5-5x the A + B bytes for 8
// and 16 rows alike (1.22 / 1.36 GB), so the group size does not act through the
// wave's L2 footprint alone. Hence: 16 rows, or 32 when the output has at most 16
// tile-columns. Overridable for measurements.
std::atomic<int> g_gemm_group_rows_override{0};

int gemm_group_rows(int n_tiles) {
    const int forced = g_gemm_group_rows_override.load(std::memory_order_relaxed);
    if (forced > 0) return forced;
    return n_tiles <= 16 ? 32 : tk::gemm::kGroupM;
}

// Tiling of a GEMM on single-CTA or CTA-pair tiles: tile width, K splits.
struct GemmPlan {
    int bn = tk::gemm::kBlockN;  // columns per tile: 256, or 128 for small-M split-K
    int n_tiles = 0;
    long long tiles = 0;
    int k_splits = 1, kb_per_split = 0;
    bool cluster_fits = false;  // every tile's cluster of k_splits CTAs is resident at once
};

// Splits K when the output has too few tiles to occupy the GPU (decode-shaped
// problems): at least 4 K blocks per split, partials at most 64 MiB. On single-CTA
// tiles the split count is then lowered, if needed, to the largest one (at most 8:
// the portable cluster size) whose tile clusters can all be resident at once, so
// the splits of a tile can reduce inside their cluster. The plan does not depend
// on how the splits are reduced.
template <int kBN>
GemmPlan plan_gemm(long long m_tiles, long long m, long long n, int k_blocks, bool may_split, int cta_group,
                   int sm_count, int device) {
    GemmPlan g;
    g.bn = kBN;
    g.n_tiles = static_cast<int>((n + kBN - 1) / kBN);
    g.tiles = m_tiles * g.n_tiles;
    g.kb_per_split = k_blocks;
    if (may_split && g.tiles < sm_count / 2 && k_blocks >= 8) {
        int splits = static_cast<int>(sm_count / g.tiles);
        if (splits > k_blocks / 4) splits = k_blocks / 4;
        while (splits > 1 && static_cast<long long>(splits) * m * n * 4 > (64LL << 20)) --splits;
        if (splits > 1) {
            g.kb_per_split = (k_blocks + splits - 1) / splits;
            g.k_splits = (k_blocks + g.kb_per_split - 1) / g.kb_per_split;
        }
    }
    if (g.k_splits > 1 && cta_group == 1) {
        for (int s = g.k_splits < 8 ? g.k_splits : 8; s >= 2 && !g.cluster_fits; --s) {
            const int kb_per = (k_blocks + s - 1) / s;
            const int splits = (k_blocks + kb_per - 1) / kb_per;
            if (splits >= 2 && g.tiles <= split_cluster_capacity<kBN>(device, splits)) {
                g.kb_per_split = kb_per;
                g.k_splits = splits;
                g.cluster_fits = true;
            }
        }
    }
    return g;
}

// Small-M GEMM (M <= 64): sets skinny_kernel's shared-memory limit on `device`, once.
cudaError_t skinny_configure(int device) {
    static std::atomic<bool> configured[tk::host::kMaxDevices];
    if (configured[device].load(std::memory_order_acquire)) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(tk::gemm::skinny_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tk::gemm::kSkinnySmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tk::gemm::skinny_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 tk::gemm::kSkinnySmemBytes);
    if (e != cudaSuccess) return e;
    configured[device].store(true, std::memory_order_release);
    return cudaSuccess;
}

// How many clusters of `splits` CTAs of skinny_kernel can be resident at once on
// `device` (cached; 0 when the query fails). skinny_configure must have succeeded.
int skinny_cluster_capacity(int device, int splits) {
    static std::atomic<int> cache[tk::host::kMaxDevices][9];
    int v = cache[device][splits].load(std::memory_order_acquire);
    if (v != 0) return v < 0 ? 0 : v;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(splits));
    cfg.blockDim = dim3(tk::gemm::kThreads);
    cfg.dynamicSmemBytes = tk::gemm::kSkinnySmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, tk::gemm::skinny_kernel<true>, &cfg) != cudaSuccess) {
        static_cast<void>(cudaGetLastError());
        clusters = 0;
    }
    cache[device][splits].store(clusters > 0 ? clusters : -1, std::memory_order_release);
    return clusters;
}

std::atomic<int> g_gemm_splitk_mode{0};  // 0 = in-cluster reduction where it fits, 1 = always the separate kernel
std::atomic<int> g_gemm_small_m{1};       // 1 = operand-swapped kernel for m <= 64, 0 = 128-row tiles

// C = A B for m <= 64 on skinny_kernel: one CTA per (128-column tile, K split), two
// CTAs per SM. Splits fill the GPU (at most 8, at least 2 K blocks each) and are
// summed in split order: inside the tile's cluster when every cluster can be
// resident at once (and the reduction mode allows it), else by splitk_reduce_kernel.
cudaError_t skinny_gemm(int m, int n, int k, const void* a, long long lda, const void* b, long long ldb, float* c,
                        long long ldc, bool c_vec4, int device, int sm_count, cudaStream_t stream) {
    using namespace tk::gemm;
    cudaError_t err = skinny_configure(device);
    if (err != cudaSuccess) return err;
    const int n_tiles = (n + kSkinnyBN - 1) / kSkinnyBN;
    const int k_blocks = (k + kBlockK - 1) / kBlockK;
    int splits = 1;
    const int want = (2 * sm_count) / n_tiles;
    if (want > 1 && k_blocks >= 4) splits = want < 8 ? want : 8;
    if (splits > k_blocks / 2) splits = k_blocks / 2 > 1 ? k_blocks / 2 : 1;
    int kb_per = (k_blocks + splits - 1) / splits;
    splits = (k_blocks + kb_per - 1) / kb_per;
    // The split count is lowered, if needed, to the largest whose tile clusters can all be
    // resident at once; it does not depend on the reduction mode, so both forms give the
    // same bits.
    bool fits = false;
    for (int s = splits; s >= 2 && !fits; --s) {
        const int kp = (k_blocks + s - 1) / s;
        const int ss = (k_blocks + kp - 1) / kp;
        if (ss >= 2 && n_tiles <= skinny_cluster_capacity(device, ss)) {
            splits = ss;
            kb_per = kp;
            fits = true;
        }
    }
    const bool cluster = fits && g_gemm_splitk_mode.load(std::memory_order_relaxed) == 0;
    SkinnyParams p{};
    p.m = m;
    p.n = n;
    p.k = k;
    p.m_pad = (m + 15) / 16 * 16;
    p.c = c;
    p.ldc = ldc;
    p.c_vec4 = c_vec4;
    p.n_tiles = n_tiles;
    p.k_blocks = k_blocks;
    p.k_splits = splits;
    p.kb_per_split = kb_per;
    p.ws = nullptr;
    CUtensorMap mb, ma;
    const uint64_t b_dims[2] = {static_cast<uint64_t>(n), static_cast<uint64_t>(k)};
    const uint64_t b_strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t b_box[2] = {64, 64};
    const uint64_t a_dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t a_strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t a_box[2] = {64, static_cast<uint32_t>(p.m_pad)};
    if (!tk::host::make_map_f16(&mb, b, 2, b_dims, b_strides, b_box) ||
        !tk::host::make_map_f16(&ma, a, 2, a_dims, a_strides, a_box)) {
        return cudaErrorInvalidValue;
    }
    if (splits > 1 && !cluster) {
        err = tk::host::scratch_alloc(reinterpret_cast<void**>(&p.ws),
                                      static_cast<size_t>(splits) * m * n * sizeof(float), device, stream);
        if (err != cudaSuccess) return err;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * splits));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSkinnySmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster ? 1 : 0;
    err = cluster ? cudaLaunchKernelEx(&cfg, skinny_kernel<true>, mb, ma, p)
                  : cudaLaunchKernelEx(&cfg, skinny_kernel<false>, mb, ma, p);
    if (p.ws != nullptr) {
        if (err == cudaSuccess) {
            const long long quads = static_cast<long long>(m) * (n / 4);
            const int blocks = static_cast<int>(quads / 256 + 1 < 4 * sm_count ? quads / 256 + 1 : 4 * sm_count);
            cudaLaunchConfig_t rcfg{};
            rcfg.gridDim = dim3(static_cast<unsigned>(blocks));
            rcfg.blockDim = dim3(256);
            rcfg.stream = stream;
            cudaLaunchAttribute rattr[1];
            rattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            rattr[0].val.programmaticStreamSerializationAllowed = 1;
            rcfg.attrs = rattr;
            rcfg.numAttrs = 1;
            err = cudaLaunchKernelEx(&rcfg, splitk_reduce_kernel, static_cast<const float*>(p.ws), splits, m, n, c, ldc,
                                     c_vec4);
        }
        cudaFreeAsync(p.ws, stream);
    }
    return err;
}

// Destinations of the multi-GPU gathered GEMM: rank `rank` of `count` writes its m
// rows at row rank * m of each buffer (count == 0: an ordinary GEMM into c).
struct Gather {
    float* const* bufs = nullptr;
    int count = 0;
    int rank = 0;
};

cudaError_t gemm_impl(int m, int n, int k, const void* a, int lda, const void* b, int ldb, float* c,
                      int ldc, float* row_max, float* row_sum, float* probs, int ldp, cudaStream_t stream,
                      Gather gather = Gather{}) {
    const bool softmax = probs != nullptr;
    const bool stats = row_max != nullptr || row_sum != nullptr || softmax;
    const bool gathered = gather.count > 0;
    if (a == nullptr || b == nullptr || c == nullptr || m <= 0 || n <= 0 || k <= 0 || m % 16 != 0 ||
        n % 16 != 0 || k % 16 != 0 || lda < k || ldb < n || ldc < n) {
        return cudaErrorInvalidValue;
    }
    if (softmax) {
        if (ldp < n) return cudaErrorInvalidValue;
        // P either replaces C exactly (in place) or lies entirely outside it.
        const size_t c_bytes = (static_cast<size_t>(m - 1) * ldc + n) * sizeof(float);
        const size_t p_bytes = (static_cast<size_t>(m - 1) * ldp + n) * sizeof(float);
        if (!(probs == c && ldp == ldc) && tk::host::ranges_overlap(probs, p_bytes, c, c_bytes))
            return cudaErrorInvalidValue;
    }
    if (stats && !softmax &&
        (row_max == nullptr || row_sum == nullptr ||
         tk::host::ranges_overlap(row_max, sizeof(float) * m, row_sum, sizeof(float) * m))) {
        return cudaErrorInvalidValue;
    }
    bool gather_vec4 = true;
    if (gathered) {
        for (int r = 0; r < gather.count; ++r) gather_vec4 = gather_vec4 && aligned(gather.bufs[r], 16);
        gather_vec4 = gather_vec4 && ldc % 4 == 0;
    }
    int sm_count = 0, device = 0;
    cudaError_t err = current_device(&device, &sm_count);
    if (err != cudaSuccess) return err;
    static_cast<void>(cudaGetLastError());

    // Operands whose rows TMA cannot address (row pitch not a multiple of 16
    // bytes, or a base that is not 16-byte aligned) are first copied into dense
    // stream-ordered buffers.
    const void* a_use = a;
    const void* b_use = b;
    long long lda_use = lda, ldb_use = ldb;
    void* a_tmp = nullptr;
    void* b_tmp = nullptr;
    if (!aligned(a, 16) || lda % 8 != 0) {
        err = tk::host::scratch_alloc(&a_tmp, static_cast<size_t>(m) * k * 2, device, stream);
        if (err != cudaSuccess) return err;
        tk::gemm::repack_f16_kernel<<<1024, 256, 0, stream>>>(static_cast<const uint16_t*>(a), lda,
                                                              static_cast<uint16_t*>(a_tmp), m, k);
        a_use = a_tmp;
        lda_use = k;
    }
    if (!aligned(b, 16) || ldb % 8 != 0) {
        err = tk::host::scratch_alloc(&b_tmp, static_cast<size_t>(k) * n * 2, device, stream);
        if (err != cudaSuccess) {
            if (a_tmp) cudaFreeAsync(a_tmp, stream);
            return err;
        }
        tk::gemm::repack_f16_kernel<<<1024, 256, 0, stream>>>(static_cast<const uint16_t*>(b), ldb,
                                                              static_cast<uint16_t*>(b_tmp), k, n);
        b_use = b_tmp;
        ldb_use = n;
    }

    int cta_group = g_gemm_cta_group_override.load(std::memory_order_relaxed);
    // Up to 64 rows (decode-shaped): the operand-swapped kernel, unless CTA pairs are forced.
    if (m <= tk::gemm::kSkinnyMaxM && !stats && !gathered && cta_group != 2 &&
        g_gemm_small_m.load(std::memory_order_relaxed) != 0) {
        err = skinny_gemm(m, n, k, a_use, lda_use, b_use, ldb_use, c, ldc, aligned(c, 16) && ldc % 4 == 0, device,
                          sm_count, stream);
        if (a_tmp) cudaFreeAsync(a_tmp, stream);
        if (b_tmp) cudaFreeAsync(b_tmp, stream);
        if (err != cudaSuccess) return err;
        return cudaGetLastError();
    }
    if (cta_group == 0) {
        const long long big_tiles = ((m + 255LL) / 256) * ((n + 255LL) / 256);
        cta_group = big_tiles >= sm_count / 2 ? 2 : 1;
    }

    const int tile_m = tk::gemm::kBlockM * cta_group;
    const long long m_tiles = (m + tile_m - 1) / tile_m;
    const int k_blocks = (k + tk::gemm::kBlockK - 1) / tk::gemm::kBlockK;
    const bool may_split = !stats && !gathered;
    GemmPlan plan = plan_gemm<256>(m_tiles, m, n, k_blocks, may_split, cta_group, sm_count, device);
    // Small split-K problems that leave more than half of the SMs idle take
    // 128-column tiles when these put more CTAs to work. Measured per call, back to
    // back: 512^3 14.5 -> 11.5 us (16 -> 32 CTAs), 48 x 784 x 2048 10.3 -> 8.8 us
    // (32 -> 56 CTAs); 16 x 4096 x 4096 (96 CTAs on 256-column tiles) was slower
    // on 128 CTAs of 128 columns, 11.8 vs 11.3 us.
    if (plan.cluster_fits && plan.tiles * plan.k_splits <= sm_count / 2) {
        const GemmPlan narrow = plan_gemm<128>(m_tiles, m, n, k_blocks, may_split, cta_group, sm_count, device);
        if (narrow.cluster_fits && narrow.tiles * narrow.k_splits > plan.tiles * plan.k_splits) plan = narrow;
    }
    if (plan.tiles > INT_MAX / (plan.k_splits > 0 ? plan.k_splits : 1)) {
        if (a_tmp) cudaFreeAsync(a_tmp, stream);
        if (b_tmp) cudaFreeAsync(b_tmp, stream);
        return cudaErrorInvalidValue;
    }

    CUtensorMap ma, mb;
    const uint64_t a_dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t a_strides[1] = {static_cast<uint64_t>(lda_use) * 2};
    const uint32_t a_box[2] = {64, 128};
    const uint64_t b_dims[2] = {static_cast<uint64_t>(n), static_cast<uint64_t>(k)};
    const uint64_t b_strides[1] = {static_cast<uint64_t>(ldb_use) * 2};
    const uint32_t b_box[2] = {64, 64};
    if (!tk::host::make_map_f16(&ma, a_use, 2, a_dims, a_strides, a_box) ||
        !tk::host::make_map_f16(&mb, b_use, 2, b_dims, b_strides, b_box)) {
        if (a_tmp) cudaFreeAsync(a_tmp, stream);
        if (b_tmp) cudaFreeAsync(b_tmp, stream);
        return cudaErrorInvalidValue;
    }

    tk::gemm::Params p{};
    p.m = m;
    p.n = n;
    p.k = k;
    p.c = c;
    p.ldc = ldc;
    p.c_vec4 = gathered ? gather_vec4 : aligned(c, 16) && ldc % 4 == 0;
    if (gathered) {
        p.n_dst = gather.count;
        for (int r = 0; r < gather.count; ++r) p.dst[r] = gather.bufs[r];
        p.dst_row0 = static_cast<long long>(gather.rank) * m;
    }
    p.m_tiles = static_cast<int>(m_tiles);
    p.n_tiles = plan.n_tiles;
    p.group_m = gemm_group_rows(p.n_tiles);
    p.k_blocks = k_blocks;
    p.k_splits = plan.k_splits;
    p.kb_per_split = plan.kb_per_split;
    const long long tiles = plan.tiles;
    const bool narrow = plan.bn == 128;
    // Both reductions add the same splits in the same order: the results do not
    // depend on the mode.
    const bool cluster_reduce = plan.cluster_fits && g_gemm_splitk_mode.load(std::memory_order_relaxed) == 0;
    p.num_tiles = static_cast<int>(tiles) * p.k_splits;
    p.ws = nullptr;
    if (p.k_splits > 1 && !cluster_reduce) {
        err = tk::host::scratch_alloc(reinterpret_cast<void**>(&p.ws),
                                      static_cast<size_t>(p.k_splits) * m * n * sizeof(float), device, stream);
        if (err != cudaSuccess) {
            if (a_tmp) cudaFreeAsync(a_tmp, stream);
            if (b_tmp) cudaFreeAsync(b_tmp, stream);
            return err;
        }
    }

    float* partial = nullptr;
    if (stats) {
        err = tk::host::scratch_alloc(reinterpret_cast<void**>(&partial),
                                      static_cast<size_t>(m) * p.n_tiles * sizeof(float2), device, stream);
        if (err != cudaSuccess) {
            if (a_tmp) cudaFreeAsync(a_tmp, stream);
            if (b_tmp) cudaFreeAsync(b_tmp, stream);
            return err;
        }
    }
    p.partial = partial;

    using tk::gemm::kStatsMaxSum;
    using tk::gemm::kStatsNone;
    using tk::gemm::kStatsSoftmax;
    using tk::gemm::kEpiGather;
    if (cluster_reduce) {
        err = narrow ? launch_gemm_split_cluster<128>(ma, mb, p, stream)
                     : launch_gemm_split_cluster<256>(ma, mb, p, stream);
    } else if (narrow) {
        err = launch_gemm_kernel<1, kStatsNone, 128>(ma, mb, p, device, sm_count, stream);
    } else if (cta_group == 2) {
        err = gathered ? launch_gemm_kernel<2, kEpiGather>(ma, mb, p, device, sm_count, stream)
              : softmax ? launch_gemm_kernel<2, kStatsSoftmax>(ma, mb, p, device, sm_count, stream)
              : stats   ? launch_gemm_kernel<2, kStatsMaxSum>(ma, mb, p, device, sm_count, stream)
                        : launch_gemm_kernel<2, kStatsNone>(ma, mb, p, device, sm_count, stream);
    } else {
        err = gathered ? launch_gemm_kernel<1, kEpiGather>(ma, mb, p, device, sm_count, stream)
              : softmax ? launch_gemm_kernel<1, kStatsSoftmax>(ma, mb, p, device, sm_count, stream)
              : stats   ? launch_gemm_kernel<1, kStatsMaxSum>(ma, mb, p, device, sm_count, stream)
                        : launch_gemm_kernel<1, kStatsNone>(ma, mb, p, device, sm_count, stream);
    }
    if (softmax && err == cudaSuccess) {
        const bool vec4 = aligned(c, 16) && ldc % 4 == 0 && aligned(probs, 16) && ldp % 4 == 0;
        const int warps_needed = (m + 7) / 8;  // 8 rows (warps) per block
        const int blocks = warps_needed < 8 * sm_count ? warps_needed : 8 * sm_count;
        tk::gemm::rowsoftmax_apply_kernel<<<blocks, 256, 0, stream>>>(
            reinterpret_cast<const float2*>(partial), m, n, p.n_tiles, c, ldc, probs, ldp, vec4);
    } else if (stats && err == cudaSuccess) {
        tk::gemm::rowstats_finish_kernel<<<(m + 255) / 256, 256, 0, stream>>>(
            reinterpret_cast<const float2*>(partial), m, p.n_tiles, row_max, row_sum);
    }
    if (p.k_splits > 1 && !cluster_reduce) {
        if (err == cudaSuccess) {
            const long long quads = static_cast<long long>(m) * (n / 4);
            const int blocks = static_cast<int>(quads / 256 + 1 < 4 * sm_count ? quads / 256 + 1 : 4 * sm_count);
            // Programmatic dependent launch: the reduction's launch overlaps the GEMM's tail.
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(static_cast<unsigned>(blocks));
            cfg.blockDim = dim3(256);
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            err = cudaLaunchKernelEx(&cfg, tk::gemm::splitk_reduce_kernel, static_cast<const float*>(p.ws), p.k_splits,
                                     m, n, c, static_cast<long long>(ldc), p.c_vec4);
        }
        cudaFreeAsync(p.ws, stream);
    }
    if (partial) cudaFreeAsync(partial, stream);
    if (a_tmp) cudaFreeAsync(a_tmp, stream);
    if (b_tmp) cudaFreeAsync(b_tmp, stream);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Fused row-statistics GEMM without allocation
// ---------------------------------------------------------------------------

// Scratch of tk_gemm_f16_f16_f32_nn_rowstats_noalloc: one (max, sum) pair per
// (row, 256-column tile). Every GPU that loads the library holds it until exit.
// In host code this name only stands for the array: its device address comes
// from cudaGetSymbolAddress, looked up once per device below.
static __device__ __align__(256) float2 g_rowstats_noalloc_scratch[TK_GEMM_ROWSTATS_NOALLOC_MAX_PARTIALS];

std::mutex g_noalloc_mutex;
float2* g_noalloc_scratch_ptr[tk::host::kMaxDevices] = {};

// Device address of the scratch array on `device`, which must be current.
cudaError_t noalloc_scratch(int device, float2** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_scratch_ptr[device] == nullptr) {
        void* ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_rowstats_noalloc_scratch);
        if (err != cudaSuccess) return err;
        g_noalloc_scratch_ptr[device] = static_cast<float2*>(ptr);
    }
    *out = g_noalloc_scratch_ptr[device];
    return cudaSuccess;
}

cudaError_t gemm_rowstats_noalloc(int m, int n, int k, const void* a, int lda, const void* b, int ldb,
                                  float* c, int ldc, float* row_max, float* row_sum,
                                  cudaStream_t stream) {
    if (a == nullptr || b == nullptr || c == nullptr || row_max == nullptr || row_sum == nullptr ||
        m <= 0 || n <= 0 || k <= 0 || m % 16 != 0 || n % 16 != 0 || k % 16 != 0 || lda < k ||
        ldb < n || ldc < n ||
        tk::host::ranges_overlap(row_max, sizeof(float) * m, row_sum, sizeof(float) * m)) {
        return cudaErrorInvalidValue;
    }
    const long long n_tiles = (n + tk::gemm::kBlockN - 1) / tk::gemm::kBlockN;
    if (static_cast<long long>(m) * n_tiles > static_cast<long long>(TK_GEMM_ROWSTATS_NOALLOC_MAX_PARTIALS))
        return cudaErrorNotSupported;  // more partials than the built-in scratch holds
    if (!aligned(a, 16) || lda % 8 != 0 || !aligned(b, 16) || ldb % 8 != 0)
        return cudaErrorNotSupported;  // would need a repacking copy, i.e. an allocation
    int sm_count = 0, device = 0;
    cudaError_t err = current_device(&device, &sm_count);
    if (err != cudaSuccess) return err;
    static_cast<void>(cudaGetLastError());
    float2* scratch = nullptr;
    err = noalloc_scratch(device, &scratch);
    if (err != cudaSuccess) return err;

    int cta_group = g_gemm_cta_group_override.load(std::memory_order_relaxed);
    if (cta_group == 0) {
        const long long big_tiles = ((m + 255LL) / 256) * ((n + 255LL) / 256);
        cta_group = big_tiles >= sm_count / 2 ? 2 : 1;
    }
    CUtensorMap ma, mb;
    const uint64_t a_dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t a_strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t a_box[2] = {64, 128};
    const uint64_t b_dims[2] = {static_cast<uint64_t>(n), static_cast<uint64_t>(k)};
    const uint64_t b_strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t b_box[2] = {64, 64};
    if (!tk::host::make_map_f16(&ma, a, 2, a_dims, a_strides, a_box) ||
        !tk::host::make_map_f16(&mb, b, 2, b_dims, b_strides, b_box)) {
        return cudaErrorInvalidValue;
    }
    tk::gemm::Params p{};
    p.m = m;
    p.n = n;
    p.k = k;
    p.c = c;
    p.ldc = ldc;
    p.c_vec4 = aligned(c, 16) && ldc % 4 == 0;
    const int tile_m = tk::gemm::kBlockM * cta_group;
    p.m_tiles = (m + tile_m - 1) / tile_m;
    p.n_tiles = static_cast<int>(n_tiles);
    p.group_m = gemm_group_rows(p.n_tiles);
    p.k_blocks = (k + tk::gemm::kBlockK - 1) / tk::gemm::kBlockK;
    p.num_tiles = p.m_tiles * p.n_tiles;
    p.k_splits = 1;
    p.kb_per_split = p.k_blocks;
    p.ws = nullptr;
    // Every (row < m, tile) pair is written by the GEMM epilogue before the
    // finishing pass reads it, so nothing left by an earlier call is used. The one
    // exception is a GEMM that gave up on a bounded wait: it records a fault in the
    // status word, and the finishing pass then writes NaN rather than combine pairs
    // an earlier call may have left.
    p.partial = reinterpret_cast<float*>(scratch);
    err = cta_group == 2 ? launch_gemm_kernel<2, tk::gemm::kStatsMaxSum>(ma, mb, p, device, sm_count, stream)
                         : launch_gemm_kernel<1, tk::gemm::kStatsMaxSum>(ma, mb, p, device, sm_count, stream);
    if (err != cudaSuccess) return err;
    tk::gemm::rowstats_finish_kernel<<<(m + 255) / 256, 256, 0, stream>>>(scratch, m, p.n_tiles, row_max,
                                                                         row_sum);
    return cudaGetLastError();
}

}  // namespace

extern "C" {

cudaError_t tk_gemm_f16_f16_f32_nn(int m, int n, int k, const void* a, int lda, const void* b,
                                   int ldb, float* c, int ldc, cudaStream_t stream) {
    return gemm_impl(m, n, k, a, lda, b, ldb, c, ldc, nullptr, nullptr, nullptr, 0, stream);
}

cudaError_t tk_gemm_f16_f16_f32_nn_rowstats(int m, int n, int k, const void* a, int lda,
                                            const void* b, int ldb, float* c, int ldc,
                                            float* row_max, float* row_sum, cudaStream_t stream) {
    if (row_max == nullptr || row_sum == nullptr) return cudaErrorInvalidValue;
    return gemm_impl(m, n, k, a, lda, b, ldb, c, ldc, row_max, row_sum, nullptr, 0, stream);
}

cudaError_t tk_gemm_f16_f16_f32_nn_rowstats_noalloc(int m, int n, int k, const void* a, int lda,
                                                    const void* b, int ldb, float* c, int ldc,
                                                    float* row_max, float* row_sum,
                                                    cudaStream_t stream) {
    return gemm_rowstats_noalloc(m, n, k, a, lda, b, ldb, c, ldc, row_max, row_sum, stream);
}

cudaError_t tk_gemm_f16_f16_f32_nn_rowsoftmax(int m, int n, int k, const void* a, int lda,
                                              const void* b, int ldb, float* c, int ldc, float* probs,
                                              int ldp, cudaStream_t stream) {
    if (probs == nullptr) return cudaErrorInvalidValue;
    return gemm_impl(m, n, k, a, lda, b, ldb, c, ldc, nullptr, nullptr, probs, ldp, stream);
}

cudaError_t tk_gemm_f16_f16_f32_nn_gather(int m, int n, int k, const void* a, int lda, const void* b,
                                          int ldb, float* const* c_ranks, int n_ranks, int rank, int ldc,
                                          cudaStream_t stream) {
    if (c_ranks == nullptr || n_ranks < 1 || n_ranks > tk::gemm::kMaxGatherRanks || rank < 0 || rank >= n_ranks)
        return cudaErrorInvalidValue;
    for (int r = 0; r < n_ranks; ++r)
        if (c_ranks[r] == nullptr) return cudaErrorInvalidValue;
    if (m <= 0 || static_cast<long long>(n_ranks) * m > INT_MAX) return cudaErrorInvalidValue;
    Gather g;
    g.bufs = c_ranks;
    g.count = n_ranks;
    g.rank = rank;
    float* local = c_ranks[rank] + static_cast<size_t>(rank) * m * static_cast<size_t>(ldc > 0 ? ldc : 0);
    return gemm_impl(m, n, k, a, lda, b, ldb, local, ldc, nullptr, nullptr, nullptr, 0, stream, g);
}

cudaError_t tk_ipc_alloc(size_t bytes, void** ptr, void* handle) {
    if (ptr == nullptr || handle == nullptr || bytes == 0) return cudaErrorInvalidValue;
    cudaError_t err = cudaMalloc(ptr, bytes);
    if (err != cudaSuccess) return err;
    err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
    if (err != cudaSuccess) {
        static_cast<void>(cudaFree(*ptr));
        *ptr = nullptr;
    }
    return err;
}

cudaError_t tk_ipc_open(const void* handle, void** ptr) {
    if (ptr == nullptr || handle == nullptr) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

cudaError_t tk_ipc_close(void* ptr) {
    if (ptr == nullptr) return cudaErrorInvalidValue;
    return cudaIpcCloseMemHandle(ptr);
}

cudaError_t tk_ipc_free(void* ptr) {
    if (ptr == nullptr) return cudaErrorInvalidValue;
    return cudaFree(ptr);
}

int tk_gemm_set_cta_group(int cta_group) {
    if (cta_group < 0 || cta_group > 2) return g_gemm_cta_group_override.load();
    return g_gemm_cta_group_override.exchange(cta_group);
}

int tk_attention_set_cta_group(int cta_group) {
    // 1 (or 0, the default): the single-CTA kernel; 2: the CTA-pair kernel where it applies.
    if (cta_group < 0 || cta_group > 2) return tk::attn::cta_group_knob().load();
    return tk::attn::cta_group_knob().exchange(cta_group == 2 ? 2 : 1);
}

int tk_gemm_set_group_rows(int rows) {
    if (rows < 0 || rows > 4096) return g_gemm_group_rows_override.load();
    return g_gemm_group_rows_override.exchange(rows);
}

int tk_gemm_set_small_m(int mode) {
    if (mode != 0 && mode != 1) return g_gemm_small_m.load();
    return g_gemm_small_m.exchange(mode);
}

int tk_gemm_set_splitk_reduce(int mode) {
    if (mode != 0 && mode != 1) return g_gemm_splitk_mode.load();
    return g_gemm_splitk_mode.exchange(mode);
}

cudaError_t tk_tile_row_sum_f32(const float* tiles, size_t n_tiles, float* out, cudaStream_t stream) {
    return rowops(tiles, n_tiles, out, nullptr, nullptr, nullptr, false, stream);
}

cudaError_t tk_tile_row_max_f32(const float* tiles, size_t n_tiles, float* out, cudaStream_t stream) {
    return rowops(tiles, n_tiles, nullptr, out, nullptr, nullptr, false, stream);
}

cudaError_t tk_tile_row_softmax_f32(const float* tiles, size_t n_tiles, float* out,
                                    cudaStream_t stream) {
    return rowops(tiles, n_tiles, nullptr, nullptr, out, nullptr, true, stream);
}

cudaError_t tk_tile_row_softmax_causal_f32(const float* tiles, size_t n_tiles, float* out,
                                           cudaStream_t stream) {
    return rowops(tiles, n_tiles, nullptr, nullptr, nullptr, out, true, stream);
}

cudaError_t tk_tile_row_ops_f32(const float* tiles, size_t n_tiles, float* row_sum, float* row_max,
                                float* softmax, float* softmax_causal, cudaStream_t stream) {
    return rowops(tiles, n_tiles, row_sum, row_max, softmax, softmax_causal, false, stream);
}

cudaError_t tk_attention_forward_16x16(const void* q, const void* k, const void* v, float* out,
                                       cudaStream_t stream) {
    return tk::attn::attention_entry(q, k, v, out, 1, 1, 1, 16, 16, 0.25f, 0, true, stream);
}

cudaError_t tk_attention_forward_16x16_causal(const void* q, const void* k, const void* v,
                                              float* out, cudaStream_t stream) {
    return tk::attn::attention_entry(q, k, v, out, 1, 1, 1, 16, 16, 0.25f, 1, true, stream);
}

cudaError_t tk_attention_forward_f16(const void* q, const void* k, const void* v, float* out,
                                     int batch, int heads, int seq, int head_dim, float scale,
                                     int causal, cudaStream_t stream) {
    return tk::attn::attention_entry(q, k, v, out, batch, heads, heads, seq, head_dim, scale, causal, false,
                                     stream);
}

cudaError_t tk_attention_forward_gqa_f16(const void* q, const void* k, const void* v, float* out,
                                         int batch, int heads_q, int heads_kv, int seq, int head_dim,
                                         float scale, int causal, cudaStream_t stream) {
    return tk::attn::attention_entry(q, k, v, out, batch, heads_q, heads_kv, seq, head_dim, scale, causal,
                                     false, stream);
}

cudaError_t tk_device_status(uint32_t* status, int clear) {
    if (status == nullptr) return cudaErrorInvalidValue;
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return err;
    unsigned int value = 0;
    err = cudaMemcpyFromSymbol(&value, tk::g_tk_status, sizeof(value));
    if (err != cudaSuccess) return err;
    if (clear) {
        const unsigned int zero = 0;
        err = cudaMemcpyToSymbol(tk::g_tk_status, &zero, sizeof(zero));
        if (err != cudaSuccess) return err;
    }
    *status = value;
    return cudaSuccess;
}

cudaError_t tk_scratch_pool_bytes(int device, uint64_t* reserved, uint64_t* used) {
    if (reserved == nullptr || used == nullptr) return cudaErrorInvalidValue;
    if (device < 0 || device >= tk::host::kMaxDevices) return cudaErrorInvalidDevice;
    return tk::host::scratch_pool_bytes(device, reserved, used);
}

int tk_abi_version(void) { return kAbiVersion; }

}  // extern "C"
