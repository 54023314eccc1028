// attention.cuh — attention forward, softmax(Q K^T * scale) V, on sm_100a.
//
// Generalises the one-tile kernel of ThunderKittens-SM7x (src/attention.cu:10-60,
// one 16 x 16 tile, scale 1/4, one warp) to [batch, heads, seq, head_dim].
// Probabilities are rounded to binary16 (nearest even) before the PV product,
// as in src/attention.cu:43-47.
//
// Layout in HBM: Q, K, V are [B*H, S, D] binary16, out is [B*H, S, D] FP32.
// Each CTA owns one (batch, head) and two consecutive 128-row query tiles; it
// streams 128-key blocks of K and V through a four-slot shared-memory ring
// (TMA, 128-byte swizzle, D padded to a multiple of 64 with TMA zero fill).
//
// Tensor memory (512 columns): tile g uses S_g = cols [256g, 256g + 128) for the
// FP32 scores and O_g = cols [256g + 128, 256g + 256) for the FP32 output
// accumulator. Its softmax warpgroup reads S_g, writes the binary16
// probabilities back over the first 64 columns of S_g, and the MMA warp
// consumes them directly from TMEM (tcgen05.mma with A in tensor memory).
//
// MMA issue order per key block j:  S0_j, PV1_{j-1}, S1_j, PV0_j.
// While the tensor core runs PV1_{j-1} and S1_j, warpgroup 0 does the softmax
// of S0_j, and vice versa, so exponentials overlap matrix products. Because
// tcgen05 operations of one thread complete in order, the commit that
// announces S_g,j also guarantees PV_g,j-1 has finished: the softmax warpgroup
// may then rescale O_g in place.
//
// Rounding semantics: when the whole sequence fits one key block (S <= 128)
// the row max and sum are final before rounding, so P = rn16(exp(s - m) / l)
// exactly as the reference. For longer sequences the kernel keeps a running
// max m and rounds exp(s - m) (online softmax), divides by the running sum at
// the end, and stays inside the generalised bound
// (512*2^-23 + 2^-11 + gamma(2S)) * sum_t |V[t, c]|.
#pragma once

#include <atomic>
#include <climits>

#include "tk_host.cuh"
#include "tk_ptx.cuh"

namespace tk {
namespace attn {

// Warps 0-7: two softmax warpgroups; warpgroup 2: warp 8 TMA, warp 9 MMA, warps 10-11
// idle. Launched at 168 registers a thread (three warps share each SM sub-partition's
// 16,384 registers), warpgroup 2 then gives registers up to the softmax warpgroups:
// 128 x kRegsControl + 256 x kRegsSoftmax = 64,512 = 384 x 168, the launch's total.
constexpr int kThreads = 384;
constexpr int kRegsSoftmax = 208;
constexpr int kRegsControl = (kThreads * 168 - 256 * kRegsSoftmax) / 128 / 8 * 8;
static_assert(kRegsControl >= 24 && kRegsSoftmax % 8 == 0 && kRegsSoftmax <= 256, "setmaxnreg range");
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * 168, "register split above the launch total");
constexpr int kBlockQ = 128;
constexpr int kBlockKV = 128;
constexpr int kKvSlots = 4;
constexpr uint32_t kTmemCols = 512;
// In the unmasked fast path, one score pair in kPolyPairEvery takes exp2_poly2 on
// the FMA pipe instead of two MUFU exponentials (0: none). Measured on B200 at
// [8,32,4096,128]: every 4th / 3rd / 2nd pair gave 1061 / 1047 / 979 TFLOP/s
// against 1124 with MUFU alone at 168 registers, and every 4th / 3rd pair
// 1013-1034 / 990-1022 against 1109 with 208 registers (no spills), so the
// default is none.
#ifndef TK_ATTN_POLY_PAIR_EVERY
#define TK_ATTN_POLY_PAIR_EVERY 0
#endif
constexpr int kPolyPairEvery = TK_ATTN_POLY_PAIR_EVERY;

template <int kDPad>
struct Cfg {
    static constexpr int kTileBytes = kBlockQ * kDPad * 2;   // one Q / K / V tile
    static constexpr int kBoxes = kDPad / 64;                 // 64-column TMA boxes per tile
    static constexpr int kQOffset = 0;                        // Q0, Q1
    static constexpr int kKvOffset = 2 * kTileBytes;          // KV ring
    static constexpr int kBarOffset = kKvOffset + kKvSlots * kTileBytes;
    static constexpr int kSmemBytes = kBarOffset + 256 + 1024;
    static constexpr uint32_t kIdescS = idesc_f16_f32(128, kBlockKV, 0, 0);
    static constexpr uint32_t kIdescO = idesc_f16_f32(128, kDPad, 0, 1);
};

struct Params {
    int seq;           // S
    int head_dim;      // D (valid output columns)
    int pairs;         // ceil(S / 256): query-tile pairs per (batch, head)
    int bh;            // B * H (query heads)
    int heads_q;       // H
    int group;         // query heads per key/value head (1 = multi-head, >1 = GQA)
    int heads_kv;      // H / group
    float scale_log2;  // scale * log2(e)
    int causal;
    float* out;
    bool out_vec4;
    int num_items;      // bh * pairs work items, item w = (bh w / pairs, pair pairs - 1 - w % pairs)
    int* next_item;     // zeroed counter for dynamic scheduling, or null: item w -> CTA w % grid
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed FP32 pairs (sm_100 f32x2 arithmetic: two lanes of work per instruction).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("{\n\t.reg .b64 ra, rb, rc;\n\tmov.b64 ra, {%1, %2};\n\tmov.b64 rb, {%3, %4};\n\t"
        "mov.b64 rc, {%5, %6};\n\tfma.rn.f32x2 %0, ra, rb, rc;\n\t}"
        : "=l"(d)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
    return r;
}

__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    uint64_t d;
    asm("{\n\t.reg .b64 ra, rb;\n\tmov.b64 ra, {%1, %2};\n\tmov.b64 rb, {%3, %4};\n\t"
        "add.rn.f32x2 %0, ra, rb;\n\t}"
        : "=l"(d)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
    return r;
}

// 2^x for a pair on the FMA pipe (packed FP32 arithmetic), to move a share of the
// exponentials off the MUFU unit. x = n + f with n = rint(x) (the 1.5 * 2^23
// shifter leaves n in the low bits of t), f in [-0.5, 0.5]; 2^f from a degree-4
// polynomial with constant term 1 (least-squares fit on Chebyshev nodes, then
// reweighted towards equal ripple; max relative error 2.9e-6, far below binary16's
// half ulp 2^-11); 2^n is added to the exponent field. Inputs are clamped at -125
// so the result stays a normal float; anything that small rounds to 0 in binary16.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fmaxf(x.x, -125.0f);
    x.y = fmaxf(x.y, -125.0f);
    const float2 t = add2(x, make_float2(12582912.0f, 12582912.0f));
    const float2 n = add2(t, make_float2(-12582912.0f, -12582912.0f));
    const float2 f = fma2(n, make_float2(-1.0f, -1.0f), x);
    float2 q = fma2(make_float2(9.58281010e-3f, 9.58281010e-3f), f, make_float2(5.59064224e-2f, 5.59064224e-2f));
    q = fma2(q, f, make_float2(2.40240991e-1f, 2.40240991e-1f));
    q = fma2(q, f, make_float2(6.93124175e-1f, 6.93124175e-1f));
    q = fma2(q, f, make_float2(1.0f, 1.0f));
    return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Score of column `col` in log2 units for the masked / non-positive-scale path:
// scaled when the scale is not positive (then the exponent argument uses factor
// 1), -inf when the key is masked.
__device__ __forceinline__ float score_slow(uint32_t raw, int col, int limit, bool pos_scale, float c_in) {
    float v = __uint_as_float(raw);
    if (!pos_scale) v *= c_in;
    return col >= limit ? -INFINITY : v;
}

// Row max over the 128 scores of this thread's row (S in TMEM at s_addr), read as
// two pairs of 32-column chunks. kFast: no masked key and a positive scale.
template <bool kFast>
__device__ __forceinline__ float score_row_max(uint32_t s_addr, int limit, bool pos_scale, float c_in) {
    float mx[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) mx[t] = -INFINITY;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(s_addr + 64 * half, ra);
        tmem_ld_32x32b_x32(s_addr + 64 * half + 32, rb);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float va = kFast ? __uint_as_float(ra[i]) : score_slow(ra[i], 64 * half + i, limit, pos_scale, c_in);
            const float vb = kFast ? __uint_as_float(rb[i]) : score_slow(rb[i], 64 * half + 32 + i, limit, pos_scale, c_in);
            mx[i & 7] = fmaxf(mx[i & 7], fmaxf(va, vb));
        }
    }
    return fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
}

// Exponentials 2^(s * c_eff - m) of the row, chunk by chunk, with the next chunk's
// TMEM load in flight while the current one is computed (the single-block path
// and a non-positive scale; the others take row_exp_store128). kMode 0: write binary16 P (over
// the S columns already consumed) and return the sum; 1: only return the sum;
// 2: write binary16 P / norm (exact normalise-then-round of a single key block).
template <bool kFast, int kMode>
__device__ __forceinline__ float score_row_exp(uint32_t s_addr, int limit, bool pos_scale, float c_in,
                                               float c_eff, float neg_m, float norm) {
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
    uint32_t r[2][32];
    tmem_ld_32x32b_x32(s_addr, r[0]);
    tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        if (c < 3) tmem_ld_32x32b_x32(s_addr + 32 * (c + 1), r[(c + 1) & 1]);
        float e[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float v = kFast ? __uint_as_float(r[c & 1][i]) : score_slow(r[c & 1][i], 32 * c + i, limit, pos_scale, c_in);
            e[i] = ex2(fmaf(v, c_eff, neg_m));
            acc[i & 7] += e[i];
        }
        if constexpr (kMode != 1) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if constexpr (kMode == 2) {
                    pk[i] = pack_half2(__fdiv_rn(e[2 * i], norm), __fdiv_rn(e[2 * i + 1], norm));
                } else {
                    pk[i] = pack_half2(e[2 * i], e[2 * i + 1]);
                }
            }
            tmem_st_32x32b_x16(s_addr + 16 * c, pk);
        }
        if (c < 3) tmem_wait_ld();
    }
    return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

// Main path (positive scale, more than one key block): the thread's whole
// 128-score row comes into registers with one TMEM round trip (four loads in
// flight, one wait); masking, the max, the exponentials, their sum and the
// binary16 P are then computed from registers.
__device__ __forceinline__ void load_row128(uint32_t s_addr, uint32_t (&r)[128]) {
    tmem_ld_32x32b_x32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
    tmem_ld_32x32b_x32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
    tmem_ld_32x32b_x32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[64]));
    tmem_ld_32x32b_x32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&r[96]));
    tmem_wait_ld();
}

// Keys at column >= limit are masked: their scores become -inf.
__device__ __forceinline__ void mask_row128(uint32_t (&r)[128], int limit) {
#pragma unroll
    for (int i = 0; i < 128; ++i)
        if (i >= limit) r[i] = 0xff800000u;  // -inf
}

__device__ __forceinline__ float row_max128(const uint32_t (&r)[128]) {
    float mx[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) mx[t] = __uint_as_float(r[t]);
#pragma unroll
    for (int i = 8; i < 128; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(r[i]));
    return fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
}

// 2^(s * c - m) for the 128 scores; writes binary16 P over the first 64 columns
// (whose scores are already in registers) and returns the sum. The exponent
// arguments and the running sums use packed FP32 pairs.
__device__ __forceinline__ float row_exp_store128(uint32_t s_addr, const uint32_t (&r)[128], float c,
                                                  float neg_m) {
    float2 acc[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) acc[t] = make_float2(0.0f, 0.0f);
    const float2 c2 = make_float2(c, c);
    const float2 m2 = make_float2(neg_m, neg_m);
#pragma unroll
    for (int chunk = 0; chunk < 4; ++chunk) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int idx = 32 * chunk + 2 * i;
            const float2 a = fma2(make_float2(__uint_as_float(r[idx]), __uint_as_float(r[idx + 1])), c2, m2);
            const bool poly = kPolyPairEvery > 0 && i % (kPolyPairEvery > 0 ? kPolyPairEvery : 1) == kPolyPairEvery - 1;
            const float2 e = poly ? exp2_poly2(a) : make_float2(ex2(a.x), ex2(a.y));
            acc[i & 3] = add2(acc[i & 3], e);
            pk[i] = pack_half2(e.x, e.y);
        }
        tmem_st_32x32b_x16(s_addr + 16 * chunk, pk);
    }
    const float2 s01 = add2(acc[0], acc[1]);
    const float2 s23 = add2(acc[2], acc[3]);
    const float2 t = add2(s01, s23);
    return t.x + t.y;
}

// Moves the running reference point m_run (log2 units) for a block whose max is
// m_blk. The point only moves when the max grows by more than 8 (so unnormalised
// probabilities stay <= 2^8); otherwise O needs no rescale. The first block always
// sets it, so a single-block row uses its exact max. A row with no allowed key yet
// (only padding rows) keeps a finite point. alpha rescales O and the running sum.
__device__ __forceinline__ void next_point(float m_run, float m_blk, float& m_use, float& alpha) {
    const float m_new = fmaxf(m_run, m_blk);
    m_use = m_new > m_run + 8.0f ? m_new : m_run;
    if (m_use == -INFINITY) m_use = 0.0f;
    alpha = m_use == m_run ? 1.0f : ex2(m_run - m_use);
}

// Geometry of work item w: one (batch, head) and a pair of 128-row query tiles.
// Within a (batch, head) the items run heaviest first (later query pairs see more
// keys under causal masking), and the items of one (batch, head) are adjacent, so
// the CTAs running at one time share its K and V blocks through L2.
struct Item {
    int bh, bh_kv, q0, n_blocks, n_blocks0;
    bool has_tile1;
};

__device__ __forceinline__ Item make_item(int w, const Params& p) {
    Item it;
    const int pair = p.pairs - 1 - w % p.pairs;
    it.bh = w / p.pairs;
    // Key/value slice: query head h of batch b reads key/value head h / group.
    it.bh_kv = (it.bh / p.heads_q) * p.heads_kv + (it.bh % p.heads_q) / p.group;
    it.q0 = pair * 2 * kBlockQ;
    it.has_tile1 = it.q0 + kBlockQ < p.seq;
    const int kv_end = p.causal ? min(p.seq, it.q0 + (it.has_tile1 ? 2 : 1) * kBlockQ) : p.seq;
    it.n_blocks = (kv_end + kBlockKV - 1) / kBlockKV;
    // Causal with two tiles: the last key block starts at or after q0 + 128, past
    // every row of tile 0, so tile 0 stops one block early (it would be all masked).
    it.n_blocks0 = (p.causal && it.has_tile1) ? it.n_blocks - 1 : it.n_blocks;
    return it;
}

// Persistent: each CTA loops over work items. The TMA warp fetches the next item
// number (a counter in global memory, or a static stride when the grid covers all
// items), publishes it to the other roles through a two-entry ring in shared memory,
// and prefetches the item's Q and first K/V blocks while the previous item's last
// blocks and its output are still being processed. Barrier phases continue across
// items.
template <int kDPad>
__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const Params p) {
    using C = Cfg<kDPad>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);
    const uint32_t bars = base + C::kBarOffset;
    auto kv_full = [&](int s) { return bars + 8u * s; };
    auto kv_empty = [&](int s) { return bars + 8u * (kKvSlots + s); };
    constexpr int kB = 2 * kKvSlots;
    const uint32_t q_full = bars + 8u * kB;
    const uint32_t q_empty = bars + 8u * (kB + 1);
    auto s_full = [&](int g) { return bars + 8u * (kB + 2 + g); };
    auto p_ready = [&](int g) { return bars + 8u * (kB + 4 + g); };
    auto o_final = [&](int g) { return bars + 8u * (kB + 6 + g); };
    auto o_empty = [&](int g) { return bars + 8u * (kB + 8 + g); };
    auto item_full = [&](int s) { return bars + 8u * (kB + 10 + s); };
    auto item_empty = [&](int s) { return bars + 8u * (kB + 12 + s); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOffset + 8 * (kB + 14));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* item_info = reinterpret_cast<volatile int*>(tmem_slot + 2);  // two entries

    const uint32_t warp = warp_id();
    const uint32_t lane = lane_id();
    const bool single = p.seq <= kBlockKV;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kKvSlots; ++s) {
            mbar_init(kv_full(s), 1);
            mbar_init(kv_empty(s), 1);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int g = 0; g < 2; ++g) {
            mbar_init(s_full(g), 1);
            mbar_init(p_ready(g), 4);
            mbar_init(o_final(g), 1);
            mbar_init(o_empty(g), 4);
            mbar_init(item_full(g), 1);
            mbar_init(item_empty(g), 9);  // the MMA thread and the eight softmax warps
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc<1>(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // The register change sits inside each warpgroup's branch: ptxas sizes each
    // branch's registers by the setmaxnreg that dominates it (one placed before the
    // branches made it size all of them by the smallest).
    if (warp >= 8) {
        setmaxnreg_dec<kRegsControl>();
        if (warp == 8) {
            // ---------------- TMA producer and scheduler (one thread) ----------------
            if (lane == 0) {
                tma_prefetch_desc(&map_q);
                tma_prefetch_desc(&map_k);
                tma_prefetch_desc(&map_v);
                int slot = 0;
                uint32_t phase = 0;
                int issued = 0;
                int items = 0;
                bool ok = true;
                int w = static_cast<int>(blockIdx.x);
                for (int it_slot = 0;; it_slot ^= 1) {
                    if (items > 0) {
                        w = p.next_item != nullptr ? static_cast<int>(gridDim.x) + atomicAdd(p.next_item, 1)
                                                   : w + static_cast<int>(gridDim.x);
                    }
                    const int wi = w < p.num_items ? w : -1;
                    // Entry it_slot was last used two items ago.
                    if (items >= 2 &&
                        !mbar_wait(item_empty(it_slot), static_cast<uint32_t>((items - 2) >> 1) & 1u,
                                   kFaultProducerWait, abort_flag)) {
                        ok = false;
                        break;
                    }
                    item_info[it_slot] = wi;
                    mbar_arrive(item_full(it_slot));
                    if (wi < 0) break;
                    const Item it = make_item(wi, p);
                    // Q of the previous item is free once all its S MMAs have completed.
                    if (items > 0 &&
                        !mbar_wait(q_empty, static_cast<uint32_t>(items - 1) & 1u, kFaultProducerWait, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const int ntiles = it.has_tile1 ? 2 : 1;
                    mbar_arrive_expect_tx(q_full, ntiles * C::kTileBytes);
                    for (int g = 0; g < ntiles; ++g)
                        for (int x = 0; x < C::kBoxes; ++x)
                            tma_load_3d(base + C::kQOffset + g * C::kTileBytes + x * 16384, &map_q, q_full,
                                        x * 64, it.q0 + g * kBlockQ, it.bh);
                    ++items;
                    for (int j = 0; j < it.n_blocks && ok; ++j) {
                        for (int which = 0; which < 2; ++which) {  // K then V
                            if (!mbar_wait(kv_empty(slot), phase ^ 1u, kFaultProducerWait, abort_flag)) {
                                ok = false;
                                break;
                            }
                            const uint32_t dst = base + C::kKvOffset + slot * C::kTileBytes;
                            mbar_arrive_expect_tx(kv_full(slot), C::kTileBytes);
                            for (int x = 0; x < C::kBoxes; ++x)
                                tma_load_3d(dst + x * 16384, which == 0 ? &map_k : &map_v, kv_full(slot),
                                            x * 64, j * kBlockKV, it.bh_kv);
                            ++issued;
                            if (++slot == kKvSlots) {
                                slot = 0;
                                phase ^= 1u;
                            }
                        }
                    }
                    if (!ok) break;
                }
                if (!ok) {
                    // Let every issued load land before the CTA may exit: the last Q load
                    // and the last (up to kKvSlots) K/V loads.
                    if (items > 0) mbar_wait(q_full, static_cast<uint32_t>(items - 1) & 1u, kFaultDrainWait, nullptr);
                    int s = slot;
                    uint32_t ph = phase;
                    for (int i = 0; i < min(issued, kKvSlots); ++i) {
                        if (--s < 0) {
                            s = kKvSlots - 1;
                            ph ^= 1u;
                        }
                        mbar_wait(kv_full(s), ph, kFaultDrainWait, nullptr);
                    }
                }
            }
            __syncwarp();
        } else if (warp == 9) {
            // ---------------- MMA issuer (one thread) ----------------
            // Issue order per key block j: S0_j, PV1_{j-1}, S1_j, PV0_j. Before PV0_j the
            // thread also waits for K_{j+1}, so PV0_j and S0_{j+1} go to the tensor pipe
            // back to back: the chain PV0_j -> S0_{j+1} -> softmax 0 is the critical path.
            if (lane == 0) {
                const uint32_t q_addr[2] = {base + C::kQOffset, base + C::kQOffset + C::kTileBytes};
                auto kv_addr = [&](int slot) { return base + C::kKvOffset + slot * C::kTileBytes; };
                // The start address sits in the low 14 bits of a descriptor (16-byte units)
                // and every tile ends below 256 KiB, so a step inside a tile is a plain add
                // to the tile's base descriptor. This thread's instruction stream sets the
                // pace (a clock64 trace: ~75 cycles per MMA issued, the tensor pipe done
                // ~150 cycles after the last one of a group), so it is kept short.
                const uint64_t dq[2] = {sw128_desc(q_addr[0], 16, 1024), sw128_desc(q_addr[1], 16, 1024)};
                auto issue_s = [&](int g, uint32_t k_addr) {
                    const uint64_t dk = sw128_desc(k_addr, 16, 1024);
    #pragma unroll
                    for (int kk = 0; kk < kDPad / 16; ++kk) {
                        const uint64_t off = static_cast<uint64_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
                        mma_f16_ss<1>(tmem + 256u * g, dq[g] + off, dk + off, C::kIdescS, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(s_full(g));
                };
                auto issue_pv = [&](int g, uint32_t v_addr, bool first) {
                    const uint64_t dv = sw128_desc(v_addr, 16384, 1024);
    #pragma unroll
                    for (int kk = 0; kk < kBlockKV / 16; ++kk)
                        mma_f16_ts(tmem + 256u * g + 128u, tmem + 256u * g + kk * 8,
                                   dv + static_cast<uint64_t>((kk * 2048) >> 4), C::kIdescO,
                                   (!first || kk > 0) ? 1u : 0u);
                };
                uint32_t pr_phase[2] = {0, 0};
                int done[2] = {0, 0};  // items in which tile g has produced an output
                int kv_base = 0;       // K/V loads of the previous items
                int items = 0;
                bool ok = true;
                // The first PV of tile g in an item overwrites O_g: the softmax warps must
                // have read the previous item's O_g out of tensor memory.
                auto o_free = [&](int g) {
                    return done[g] == 0 ||
                           mbar_wait(o_empty(g), static_cast<uint32_t>(done[g] - 1) & 1u, kFaultAttnWait, abort_flag);
                };
                for (int it_slot = 0; ok; it_slot ^= 1, ++items) {
                    if (!mbar_wait(item_full(it_slot), static_cast<uint32_t>(items >> 1) & 1u, kFaultAttnWait,
                                   abort_flag))
                        break;
                    const int wi = item_info[it_slot];
                    mbar_arrive(item_empty(it_slot));
                    if (wi < 0) break;
                    const Item it = make_item(wi, p);
                    auto kv_slot = [&](int load) { return (kv_base + load) % kKvSlots; };
                    auto kv_phase = [&](int load) { return static_cast<uint32_t>((kv_base + load) / kKvSlots) & 1u; };
                    ok = mbar_wait(q_full, static_cast<uint32_t>(items) & 1u, kFaultAttnWait, abort_flag) &&
                         mbar_wait(kv_full(kv_slot(0)), kv_phase(0), kFaultAttnWait, abort_flag);
                    tc_fence_after();
                    if (ok) issue_s(0, kv_addr(kv_slot(0)));
                    const int n_blocks = it.n_blocks;
                    for (int j = 0; j < n_blocks && ok; ++j) {
                        ok = false;
                        const int k_slot = kv_slot(2 * j);
                        const int v_slot = kv_slot(2 * j + 1);
                        const int prev_v_slot = kv_slot(2 * j - 1 + kKvSlots) ;
                        const bool last = j == n_blocks - 1;
                        const bool tile0 = j < it.n_blocks0;
                        // PV1_{j-1}, then V_{j-1} is free
                        if (j > 0) {
                            if (it.has_tile1) {
                                if (!mbar_wait(p_ready(1), pr_phase[1], kFaultAttnWait, abort_flag)) break;
                                pr_phase[1] ^= 1u;
                                if (j == 1 && !o_free(1)) break;
                                tc_fence_after();
                                issue_pv(1, kv_addr(prev_v_slot), j == 1);
                            }
                            mma_commit(kv_empty(prev_v_slot));
                        }
                        // S1_j, then K_j is free. K_j was waited for before S0_j, unless
                        // tile 0 has already finished.
                        if (!tile0 && !mbar_wait(kv_full(k_slot), kv_phase(2 * j), kFaultAttnWait, abort_flag)) break;
                        if (it.has_tile1) issue_s(1, kv_addr(k_slot));
                        mma_commit(kv_empty(k_slot));
                        // After the item's last S MMA, Q may be replaced by the next item's.
                        if (last) mma_commit(q_empty);
                        // PV0_j and S0_{j+1}, back to back
                        if (!mbar_wait(kv_full(v_slot), kv_phase(2 * j + 1), kFaultAttnWait, abort_flag)) break;
                        if (tile0) {
                            const bool tile0_last = j == it.n_blocks0 - 1;
                            const int next_k_slot = kv_slot(2 * j + 2);
                            if (!tile0_last &&
                                !mbar_wait(kv_full(next_k_slot), kv_phase(2 * j + 2), kFaultAttnWait, abort_flag))
                                break;
                            if (!mbar_wait(p_ready(0), pr_phase[0], kFaultAttnWait, abort_flag)) break;
                            pr_phase[0] ^= 1u;
                            if (j == 0 && !o_free(0)) break;
                            tc_fence_after();
                            issue_pv(0, kv_addr(v_slot), j == 0);
                            if (tile0_last) {
                                mma_commit(o_final(0));
                            } else {
                                issue_s(0, kv_addr(next_k_slot));
                            }
                        }
                        if (last) {
                            // PV1_last
                            if (it.has_tile1) {
                                if (!mbar_wait(p_ready(1), pr_phase[1], kFaultAttnWait, abort_flag)) break;
                                pr_phase[1] ^= 1u;
                                if (j == 0 && !o_free(1)) break;
                                tc_fence_after();
                                issue_pv(1, kv_addr(v_slot), j == 0);
                                mma_commit(o_final(1));
                            }
                            mma_commit(kv_empty(v_slot));
                        }
                        ok = true;
                    }
                    ++done[0];
                    if (it.has_tile1) ++done[1];
                    kv_base += 2 * n_blocks;
                }
            }
            __syncwarp();
        }
    } else {
        setmaxnreg_inc<kRegsSoftmax>();
        // ---------------- softmax warpgroups (warps 0-3: tile 0, 4-7: tile 1) ----------------
        const int g = static_cast<int>(warp >> 2);
        const uint32_t quarter = warp & 3u;
        const int row_in_tile = static_cast<int>(quarter * 32 + lane);
        const uint32_t lane_bits = (quarter * 32u) << 16;
        const uint32_t s_addr = tmem + lane_bits + 256u * g;
        const uint32_t o_addr = s_addr + 128u;
        const float c_in = p.scale_log2;
        const bool pos_scale = c_in > 0.0f;
        const float c_eff = pos_scale ? c_in : 1.0f;
        uint32_t sf_phase = 0;  // s_full(g) completions seen
        uint32_t of_phase = 0;  // o_final(g) completions seen
        bool ok = true;
        for (int it_slot = 0, items = 0; ok; it_slot ^= 1, ++items) {
            if (!mbar_wait_warp(item_full(it_slot), static_cast<uint32_t>(items >> 1) & 1u, kFaultAttnWait,
                                abort_flag))
                break;
            const int wi = item_info[it_slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(item_empty(it_slot));
            if (wi < 0) break;
            const Item it = make_item(wi, p);
            if (g == 1 && !it.has_tile1) continue;
            const int q_row = it.q0 + g * kBlockQ + row_in_tile;
            float m_run = -INFINITY;  // running max, log2 units
            float l_run = 0.0f;       // running sum of exp2(s - m_run)
            const int my_blocks = g == 0 ? it.n_blocks0 : it.n_blocks;
            for (int j = 0; j < my_blocks; ++j) {
                if (!mbar_wait_warp(s_full(g), sf_phase, kFaultAttnWait, abort_flag)) {
                    ok = false;
                    break;
                }
                sf_phase ^= 1u;
                tc_fence_after();
                const int kv0 = j * kBlockKV;
                // Keys past the sequence end, and (causal) keys after this query, are masked.
                int limit = p.seq - kv0;
                if (p.causal) limit = min(limit, q_row - kv0 + 1);
                const bool need_mask = __any_sync(0xffffffffu, limit < kBlockKV);
                // Scores in log2 units are s * c. For c > 0 the max of the raw scores is
                // scaled once and each exponent argument is a single FMA; otherwise the
                // scores are scaled first. Masking runs only for blocks where some row
                // of the warp has a masked key (the choice is warp-uniform).
                const bool fast = pos_scale && !need_mask;
                float m_use, alpha, e_sum;
                if (pos_scale && !single) {
                    // Whole row in registers. Masked keys (causal diagonal, sequence
                    // tail) become -inf in place, so their exponentials are exactly 0.
                    uint32_t r[128];
                    load_row128(s_addr, r);
                    if (need_mask) mask_row128(r, limit);
                    next_point(m_run, row_max128(r) * c_eff, m_use, alpha);
                    e_sum = row_exp_store128(s_addr, r, c_eff, -m_use);
                } else {
                    const float m_raw = fast ? score_row_max<true>(s_addr, limit, pos_scale, c_in)
                                             : score_row_max<false>(s_addr, limit, pos_scale, c_in);
                    next_point(m_run, m_raw * c_eff, m_use, alpha);
                    const float neg_m = -m_use;
                    if (single) {
                        // One key block holds the whole row: sum first, then normalise and
                        // round (the exponentials are recomputed from the intact S).
                        e_sum = fast ? score_row_exp<true, 1>(s_addr, limit, pos_scale, c_in, c_eff, neg_m, 1.0f)
                                     : score_row_exp<false, 1>(s_addr, limit, pos_scale, c_in, c_eff, neg_m, 1.0f);
                        if (fast) {
                            score_row_exp<true, 2>(s_addr, limit, pos_scale, c_in, c_eff, neg_m, e_sum);
                        } else {
                            score_row_exp<false, 2>(s_addr, limit, pos_scale, c_in, c_eff, neg_m, e_sum);
                        }
                    } else {
                        e_sum = score_row_exp<false, 0>(s_addr, limit, pos_scale, c_in, c_eff, neg_m, 1.0f);
                    }
                }
                // tcgen05.ld/st are warp-collective: the rescale runs for the whole warp
                // when any of its rows needs it (alpha == 1 rows multiply by one).
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                    // Rescale the running output: PV_{j-1} has completed (in-order tcgen05).
#pragma unroll
                    for (int c = 0; c < kDPad / 16; ++c) {
                        uint32_t r[16];
                        tmem_ld_32x32b_x16(o_addr + 16 * c, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                        tmem_st_32x32b_x16(o_addr + 16 * c, r);
                    }
                }
                l_run = l_run * alpha + e_sum;
                m_run = m_use;
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_ready(g));
            }
            if (!ok || !mbar_wait_warp(o_final(g), of_phase, kFaultAttnWait, abort_flag)) {
                ok = false;
                break;
            }
            of_phase ^= 1u;
            tc_fence_after();
            const bool row_ok = q_row < p.seq;
            // Multiple rounding: one reciprocal of the row sum, then products (within
            // 2^-23 relative of a division, far inside the error bound).
            const float inv_l = single ? 1.0f : __frcp_rn(l_run);
            float* orow = p.out + (static_cast<long long>(it.bh) * p.seq + q_row) * p.head_dim;
#pragma unroll
            for (int c = 0; c < kDPad / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(o_addr + 32 * c, r);
                tmem_wait_ld();
                if (c == kDPad / 32 - 1) {
                    // O_g is in registers: the next item's first PV may overwrite it.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(o_empty(g));
                }
                if (row_ok) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int col = 32 * c + 4 * q;
                        if (col < p.head_dim) {
                            float4 v;
                            v.x = __uint_as_float(r[4 * q]) * inv_l;
                            v.y = __uint_as_float(r[4 * q + 1]) * inv_l;
                            v.z = __uint_as_float(r[4 * q + 2]) * inv_l;
                            v.w = __uint_as_float(r[4 * q + 3]) * inv_l;
                            if (p.out_vec4) {
                                __stcs(reinterpret_cast<float4*>(orow + col), v);
                            } else {
                                orow[col] = v.x;
                                orow[col + 1] = v.y;
                                orow[col + 2] = v.z;
                                orow[col + 3] = v.w;
                            }
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc<1>(tmem, kTmemCols);
    }
}

// One-tile attention (S <= 16 keys, head_dim 16): the shape of the reference's
// attention_forward_16x16 (src/attention.cu:10-60). 16 x 16 x 16 is below the
// smallest tcgen05 tile (M = 64), and a TMEM allocation, three tensor maps and a
// TMA pipeline cost several times the arithmetic, so this latency path runs on
// the FP32 pipe: one CTA of 256 threads per (batch, head), thread (i, j) owns
// score S[i][j] and output O[i][j]. Products of binary16 values are exact in
// FP32, so the dot products follow the same model as an FP32-accumulating MMA.
// Row max and sum use xor shuffles over the row's 16 lanes; P = rn16(e / l) with
// the row's final sum, the reference's normalise-then-round (src/attention.cu:38-47).
constexpr int kTileThreads = 256;

__global__ void __launch_bounds__(kTileThreads)
    attention_tile16_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                            const __half* __restrict__ v, float* __restrict__ out, int seq, int heads_q,
                            int heads_kv, int group, float scale, int causal) {
    __shared__ float qs[16][17], ks[16][17], vs[16][17], ps[16][17];
    const int t = static_cast<int>(threadIdx.x);
    const int i = t >> 4;  // query row; also the row of the element this thread loads
    const int j = t & 15;  // key index for S, output column for O
    const int bh = static_cast<int>(blockIdx.x);
    const int bh_kv = (bh / heads_q) * heads_kv + (bh % heads_q) / group;
    const long long q_base = static_cast<long long>(bh) * seq * 16;
    const long long kv_base = static_cast<long long>(bh_kv) * seq * 16;
    const bool row_valid = i < seq;
    qs[i][j] = row_valid ? __half2float(q[q_base + t]) : 0.0f;
    ks[i][j] = row_valid ? __half2float(k[kv_base + t]) : 0.0f;
    vs[i][j] = row_valid ? __half2float(v[kv_base + t]) : 0.0f;
    __syncthreads();

    float s = 0.0f;
#pragma unroll
    for (int d = 0; d < 16; ++d) s = fmaf(qs[i][d], ks[j][d], s);
    const bool masked = j >= seq || (causal && j > i);
    const float x = masked ? -INFINITY : s * scale;
    // Key 0 is never masked (seq >= 1), so every row has a finite max.
    float m = x;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o, 16));
    const float e = masked ? 0.0f : ex2((x - m) * 1.4426950408889634f);
    float l = e;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o, 16);
    ps[i][j] = __half2float(__float2half_rn(__fdiv_rn(e, l)));
    __syncthreads();

    float o_acc = 0.0f;
#pragma unroll
    for (int u = 0; u < 16; ++u) o_acc = fmaf(ps[i][u], vs[u][j], o_acc);
    if (row_valid) out[q_base + t] = o_acc;
}

__global__ void repack_kernel(const uint16_t* src, uint16_t* dst, long long count) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        dst[i] = src[i];
}

template <int kDPad>
cudaError_t launch(const void* q, const void* k, const void* v, const Params& p, int device, int grid,
                   cudaStream_t stream) {
    using Cc = Cfg<kDPad>;
    // Per-device shared-memory opt-in, done once; concurrent first calls may both
    // set the (idempotent) attribute.
    static std::atomic<bool> configured[host::kMaxDevices];
    auto kernel = attention_kernel<kDPad>;
    if (!configured[device].load(std::memory_order_acquire)) {
        cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cc::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured[device].store(true, std::memory_order_release);
    }
    CUtensorMap mq, mk, mv;
    const uint64_t dims[3] = {static_cast<uint64_t>(p.head_dim), static_cast<uint64_t>(p.seq),
                              static_cast<uint64_t>(p.bh)};
    const uint64_t dims_kv[3] = {static_cast<uint64_t>(p.head_dim), static_cast<uint64_t>(p.seq),
                                 static_cast<uint64_t>(p.bh / p.group)};
    const uint64_t strides[2] = {static_cast<uint64_t>(p.head_dim) * 2,
                                 static_cast<uint64_t>(p.head_dim) * 2 * static_cast<uint64_t>(p.seq)};
    const uint32_t box[3] = {64, 128, 1};
    if (!host::make_map_f16(&mq, q, 3, dims, strides, box) ||
        !host::make_map_f16(&mk, k, 3, dims_kv, strides, box) ||
        !host::make_map_f16(&mv, v, 3, dims_kv, strides, box)) {
        return cudaErrorInvalidValue;
    }
    kernel<<<static_cast<unsigned>(grid), kThreads, Cc::kSmemBytes, stream>>>(mq, mk, mv, p);
    return cudaSuccess;
}

namespace pair {
// CTA-pair kernel for head_dim 128 (attention_pair.cuh).
inline cudaError_t launch(const void* q, const void* k, const void* v, float* out, int bh, int heads_q,
                          int heads_kv, int seq, float scale, int causal, int device, int sm_count,
                          cudaStream_t stream);
}  // namespace pair

// Kernel choice for head_dim 128, multi-block, positive-scale problems: 1 = the
// single-CTA kernel (default: measured faster on B200, 1,140 vs 824 TFLOP/s at
// [8, 32, 4096, 128]), 2 = the CTA-pair kernel. Read by every call.
inline std::atomic<int>& cta_group_knob() {
    static std::atomic<int> knob{1};
    return knob;
}

inline cudaError_t attention_entry(const void* q, const void* k, const void* v, float* out, int batch,
                                   int heads, int heads_kv, int seq, int head_dim, float scale, int causal,
                                   bool fixed_tile, cudaStream_t stream) {
    if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) return cudaErrorInvalidValue;
    if (!fixed_tile) {
        if (batch <= 0 || heads <= 0 || heads_kv <= 0 || heads % heads_kv != 0 || seq <= 0 ||
            (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128) ||
            (causal != 0 && causal != 1) || !(scale == scale) || scale == INFINITY ||
            scale == -INFINITY) {
            return cudaErrorInvalidValue;
        }
        const long long bh = static_cast<long long>(batch) * heads;
        if (bh > INT_MAX || bh * ((seq + 255LL) / 256) > INT_MAX) return cudaErrorInvalidValue;
        const size_t elems = static_cast<size_t>(bh) * static_cast<size_t>(seq) * head_dim;
        const size_t elems_kv = elems / static_cast<size_t>(heads / heads_kv);
        if (host::ranges_overlap(out, elems * 4, q, elems * 2) ||
            host::ranges_overlap(out, elems * 4, k, elems_kv * 2) ||
            host::ranges_overlap(out, elems * 4, v, elems_kv * 2)) {
            return cudaErrorInvalidValue;
        }
    }
    int device = 0, sm_count = 0;
    cudaError_t err = host::current_device(&device, &sm_count);
    if (err != cudaSuccess) return err;
    static_cast<void>(cudaGetLastError());

    if (head_dim == 16 && seq <= 16) {
        // One tile per (batch, head): the latency path (no alignment needs beyond binary16).
        attention_tile16_kernel<<<static_cast<unsigned>(batch * heads), kTileThreads, 0, stream>>>(
            static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v), out,
            seq, heads, heads_kv, heads / heads_kv, scale, causal);
        return cudaGetLastError();
    }

    Params p{};
    p.seq = seq;
    p.head_dim = head_dim;
    p.pairs = (seq + 2 * kBlockQ - 1) / (2 * kBlockQ);
    p.bh = batch * heads;
    p.heads_q = heads;
    p.heads_kv = heads_kv;
    p.group = heads / heads_kv;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.causal = causal;
    p.out = out;
    p.out_vec4 = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    p.num_items = p.bh * p.pairs;
    p.next_item = nullptr;
    // One resident CTA per SM (shared memory and all 512 TMEM columns). With more
    // items than SMs, the CTAs take further items from a counter in stream-ordered
    // scratch memory, zeroed before the launch.
    const int grid = p.num_items < sm_count ? p.num_items : sm_count;

    // TMA needs 16-byte aligned bases; copy misaligned operands first.
    const size_t elems_q = static_cast<size_t>(p.bh) * static_cast<size_t>(seq) * head_dim;
    const size_t elems_kv = elems_q / static_cast<size_t>(p.group);
    const void* src[3] = {q, k, v};
    void* tmp[3] = {nullptr, nullptr, nullptr};
    for (int i = 0; i < 3; ++i) {
        if ((reinterpret_cast<uintptr_t>(src[i]) & 15u) != 0) {
            const size_t elems = i == 0 ? elems_q : elems_kv;
            err = host::scratch_alloc(&tmp[i], elems * 2, device, stream);
            if (err != cudaSuccess) break;
            repack_kernel<<<256, 256, 0, stream>>>(static_cast<const uint16_t*>(src[i]),
                                                   static_cast<uint16_t*>(tmp[i]),
                                                   static_cast<long long>(elems));
            src[i] = tmp[i];
        }
    }
    void* counter = nullptr;
    if (err == cudaSuccess && p.num_items > grid && !(head_dim == 128 && seq > kBlockKV && scale > 0.0f &&
                                                      cta_group_knob().load(std::memory_order_relaxed) == 2)) {
        err = host::scratch_alloc(&counter, sizeof(int), device, stream);
        if (err == cudaSuccess) err = cudaMemsetAsync(counter, 0, sizeof(int), stream);
        p.next_item = static_cast<int*>(counter);
    }
    const bool use_pair = head_dim == 128 && seq > kBlockKV && scale > 0.0f &&
                          cta_group_knob().load(std::memory_order_relaxed) == 2;
    if (err == cudaSuccess && use_pair) {
        err = pair::launch(src[0], src[1], src[2], out, p.bh, heads, heads_kv, seq, scale, causal, device, sm_count,
                           stream);
    } else if (err == cudaSuccess) {
        err = head_dim == 128 ? launch<128>(src[0], src[1], src[2], p, device, grid, stream)
                              : launch<64>(src[0], src[1], src[2], p, device, grid, stream);
    }
    if (counter != nullptr) cudaFreeAsync(counter, stream);
    for (int i = 0; i < 3; ++i)
        if (tmp[i] != nullptr) cudaFreeAsync(tmp[i], stream);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

}  // namespace attn
}  // namespace tk
