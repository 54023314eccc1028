// attention_pair.cuh — attention forward for head_dim 128 on CTA pairs
// (tcgen05.mma.cta_group::2), softmax(Q K^T * scale) V with the probabilities
// rounded to binary16 before the PV product (ThunderKittens-SM7x
// src/attention.cu:36-47, generalised to [batch, heads, seq, 128]).
//
// Why this shape. The tensor pipe keeps its dense rate (64 cycles per
// M128 x N128 x K16 MMA per SM) only while consecutive MMA groups keep one
// instruction kind and one operand major-ness; switching between A-from-shared
// and A-from-tensor-memory, or between K-major and MN-major operands, costs about
// 250 cycles per switch (measured on B200, for both CTA groups). So every MMA here
// is the same kind: both operands in shared memory, both K-major:
//   S_g  = Q_g  K_j^T   A = Q (d contiguous),       B = K   (d contiguous)
//   O_g += P_g  V_j     A = P (keys contiguous),    B = V^T (keys contiguous)
// V^T is produced by transpose_v_kernel before the launch (one extra pass over V).
// P is written to shared memory by the softmax warps instead of over S in tensor
// memory, so S_g,j+1 may be computed while the softmax of S_g,j runs: the softmax
// releases S_g,j as soon as it has the row in registers. The per-tile chain
// S -> softmax -> PV -> S of a design that aliases P onto S is gone; the softmax
// warps work back to back and the tensor pipe does the next block's S while they do.
//
// CTA pair. A cluster of two CTAs runs M = 256 MMAs issued by the even CTA: each
// CTA holds 128 query rows of a tile (A from its own shared memory), half of each
// K block (64 keys) and half of each V^T block (64 head-dim rows); the B operand
// is split between the two CTAs along N, so each CTA loads half of every K and V
// block. No TMA multicast is used.
//
// Work item: one (batch, head) and 512 query rows = two tiles of 256 rows (128 per
// CTA). Tensor memory per CTA (512 columns): S_0 [0,128), S_1 [128,256),
// O_0 [256,384), O_1 [384,512); lane = query row within the CTA's 128.
// Shared memory per CTA: Q_0, Q_1 (32 KiB each), P_0, P_1 (32 KiB each), a ring of
// six 16 KiB slots that alternately hold this CTA's half of K_j and of V^T_j.
//
// MMAs (even CTA): one issuing thread per tile, each issuing S_g,j+1 then PV_g,j for
// block j; the tensor pipe interleaves the two streams.
// Softmax of tile g (four warps per CTA, one query row per thread): wait S_g,j;
// load the row (tcgen05.ld); release S_g,j; mask, max, exponentials in registers;
// rescale O_g only when the running max grows by more than 2^8 (after PV_g,j-1 has
// completed); wait for PV_g,j-1 (P_g's buffer); store binary16 P row; announce.
//
// Rounding: exp(s - m_running) is rounded to binary16 and the output divided by
// the running sum at the end (online softmax), inside the generalised bound
// (512 * 2^-23 + 2^-11 + gamma(2S)) * sum_t |V[t, c]|. Sequences of at most one key
// block, non-positive scales and other head dims take attention_kernel.
#pragma once

#include "attention.cuh"

namespace tk {
namespace attn {
namespace pair {

constexpr int kThreads = 384;  // warps 0-7 softmax, 8 TMA, 9 TMEM + MMA (tile 0), 10 MMA (tile 1), 11 idle
constexpr int kSlots = 6;
constexpr int kTileBytes = 128 * 128 * 2;   // 128 rows x 128 binary16 (Q or P tile of one CTA)
constexpr int kSlotBytes = 64 * 128 * 2;    // half a K block (64 keys x 128) or half a V^T block (64 x 128 keys)
constexpr int kQOff = 0;
constexpr int kPOff = 2 * kTileBytes;
constexpr int kKvOff = 4 * kTileBytes;
constexpr int kBarOff = kKvOff + kSlots * kSlotBytes;
constexpr int kSmemBytes = kBarOff + 256 + 1024;  // + barriers (21 x 8 B, TMEM slot, abort flag), + alignment slack
constexpr int kRowsPerItem = 512;                 // two 256-row tiles of the pair
constexpr uint32_t kIdesc = idesc_f16_f32(256, 128, 0, 0);
// The two softmax warps of an SM sub-partition (one per tile) take turns on the MUFU
// unit for the exponentials of blocks both tiles process.
#ifndef TK_ATTN_PAIR_MUFU_TURNS
#define TK_ATTN_PAIR_MUFU_TURNS 1
#endif
constexpr bool kMufuTurns = TK_ATTN_PAIR_MUFU_TURNS != 0;
static_assert(kSmemBytes <= 232448, "shared memory above the sm_100 per-block limit");

struct PairParams {
    int seq;           // S
    int bh;            // B * H (query heads)
    int heads_q, group, heads_kv;
    float scale_log2;  // scale * log2(e), > 0
    int causal;
    float* out;        // [B*H, S, 128] FP32
    bool out_vec4;
    int quads;         // ceil(S / 512): items per (batch, head)
    int num_items;     // bh * quads
};

struct PairItem {
    int bh, bh_kv, q0;
    int nb[2];    // key blocks of tile 0 / tile 1 (0: tile absent)
    int nb_load;  // key blocks loaded: max(nb[0], nb[1])
};

// Item w: a (batch, head) slice and query rows [q0, q0 + 512). The slices are taken
// in groups of kItemGroup; inside a group the items run by quad, later (under causal
// masking heavier) quads first, slice by slice. Pairs take items w = pair, pair + pairs,
// ... (static), so the heavy and light quads spread over all pairs (simulated causal
// imbalance, max over mean: 1.06, against 1.13 when the quads of a slice are adjacent),
// while the pairs running at one time touch the K and V of about one group (32 MiB at
// S = 4096), which stays in L2.
constexpr int kItemGroup = 16;

__device__ __forceinline__ PairItem make_pair_item(int w, const PairParams& p) {
    PairItem it;
    const int per_group = kItemGroup * p.quads;
    const int g0 = (w / per_group) * kItemGroup;
    const int gsize = min(kItemGroup, p.bh - g0);
    const int within = w - (w / per_group) * per_group;
    it.bh = g0 + within % gsize;
    const int quad = p.quads - 1 - within / gsize;
    it.bh_kv = (it.bh / p.heads_q) * p.heads_kv + (it.bh % p.heads_q) / p.group;
    it.q0 = quad * kRowsPerItem;
    for (int g = 0; g < 2; ++g) {
        const int first = it.q0 + 256 * g;
        const int end = p.causal ? min(p.seq, first + 256) : p.seq;
        it.nb[g] = first < p.seq ? (end + 127) / 128 : 0;
    }
    it.nb_load = max(it.nb[0], it.nb[1]);
    return it;
}

// K-major SW128 operand of 128-byte rows: 16-row slice kk of the K dimension lives in
// box kk / 4 (box_bytes apart) at byte offset 32 * (kk % 4) of each row.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int kk, uint32_t box_bytes) {
    return sw128_desc(tile + static_cast<uint32_t>(kk >> 2) * box_bytes + static_cast<uint32_t>(kk & 3) * 32u, 16,
                      1024);
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                          const __grid_constant__ CUtensorMap map_vt, const PairParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);
    const uint32_t bars = base + kBarOff;
    auto kv_full = [&](int s) { return bars + 8u * s; };
    auto kv_empty = [&](int s) { return bars + 8u * (kSlots + s); };
    const uint32_t q_full = bars + 8u * (2 * kSlots);
    const uint32_t q_empty = bars + 8u * (2 * kSlots + 1);
    auto s_full = [&](int g) { return bars + 8u * (2 * kSlots + 2 + g); };
    auto s_free = [&](int g) { return bars + 8u * (2 * kSlots + 4 + g); };
    auto p_ready = [&](int g) { return bars + 8u * (2 * kSlots + 6 + g); };
    auto pv_done = [&](int g) { return bars + 8u * (2 * kSlots + 8 + g); };
    auto o_empty = [&](int g) { return bars + 8u * (2 * kSlots + 10 + g); };
    // MUFU turn of the two softmax warps that share an SM sub-partition (warp q of tile 0
    // and warp q + 4 of tile 1): turn(g, q) completes when tile g's warp q may run the
    // exponentials of its next block shared with the other tile.
    auto turn = [&](int g, uint32_t q) { return bars + 8u * (2 * kSlots + 12 + 4 * g + q); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kBarOff + 8 * (2 * kSlots + 20));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_id();
    const uint32_t lane = lane_id();
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster_id = static_cast<int>(blockIdx.x) >> 1;
    const int num_clusters = static_cast<int>(gridDim.x) >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(kv_full(s), 1);   // the even CTA's expect_tx; both CTAs' bytes
            mbar_init(kv_empty(s), 2);  // one MMA commit (multicast to both CTAs) per issuer
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 2);  // both issuers
        for (int g = 0; g < 2; ++g) {
            mbar_init(s_full(g), 1);
            mbar_init(s_free(g), 8);   // four softmax warps of each CTA
            mbar_init(p_ready(g), 8);
            mbar_init(pv_done(g), 1);
            mbar_init(o_empty(g), 8);
            for (uint32_t q = 0; q < 4; ++q) mbar_init(turn(g, q), 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc<2>(smem_u32(tmem_slot), 512);
        tmem_relinquish<2>();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
        setmaxnreg_dec<kRegsControl>();
        if (warp == 8 && lane == 0) {
            // ---------------- TMA producer (each CTA loads its own halves) ----------------
            tma_prefetch_desc(&map_q);
            tma_prefetch_desc(&map_k);
            tma_prefetch_desc(&map_vt);
            const uint32_t q_full_lead = mapa_shared(q_full, 0);
            const uint32_t kv_full_lead0 = mapa_shared(kv_full(0), 0);
            int slot = 0;
            uint32_t phase = 0;
            int issued = 0, items = 0;
            bool ok = true;
            for (int w = cluster_id; w < p.num_items && ok; w += num_clusters) {
                const PairItem it = make_pair_item(w, p);
                // Q of the previous item is free once its last S MMAs have completed.
                if (items > 0 &&
                    !mbar_wait(q_empty, static_cast<uint32_t>(items - 1) & 1u, kFaultProducerWait, abort_flag)) {
                    ok = false;
                    break;
                }
                const int ntiles = it.nb[1] > 0 ? 2 : 1;
                if (leader) mbar_arrive_expect_tx(q_full, 2u * ntiles * kTileBytes);
                for (int g = 0; g < ntiles; ++g)
                    for (int x = 0; x < 2; ++x)
                        tma_load_3d_pair(base + kQOff + g * kTileBytes + x * 16384, &map_q, q_full_lead, x * 64,
                                         it.q0 + 256 * g + 128 * static_cast<int>(rank), it.bh);
                ++items;
                for (int j = 0; j < it.nb_load && ok; ++j) {
                    for (int which = 0; which < 2; ++which) {  // this CTA's half of K_j, then of V^T_j
                        if (!mbar_wait(kv_empty(slot), phase ^ 1u, kFaultProducerWait, abort_flag)) {
                            ok = false;
                            break;
                        }
                        if (leader) mbar_arrive_expect_tx(kv_full(slot), 2u * kSlotBytes);
                        const uint32_t dst = base + kKvOff + slot * kSlotBytes;
                        const uint32_t fb = kv_full_lead0 + 8u * slot;
                        for (int x = 0; x < 2; ++x) {
                            if (which == 0)
                                tma_load_3d_pair(dst + x * 8192, &map_k, fb, x * 64,
                                                 128 * j + 64 * static_cast<int>(rank), it.bh_kv);
                            else
                                tma_load_3d_pair(dst + x * 8192, &map_vt, fb, 128 * j + 64 * x,
                                                 64 * static_cast<int>(rank), it.bh_kv);
                        }
                        ++issued;
                        if (++slot == kSlots) {
                            slot = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (!ok && leader) {
                // Let every load of the pair land before the CTAs may exit: the full
                // barriers count both CTAs' bytes.
                if (items > 0) mbar_wait(q_full, static_cast<uint32_t>(items - 1) & 1u, kFaultDrainWait, nullptr);
                int s = slot;
                uint32_t ph = phase;
                for (int i = 0; i < min(issued, kSlots); ++i) {
                    if (--s < 0) {
                        s = kSlots - 1;
                        ph ^= 1u;
                    }
                    mbar_wait(kv_full(s), ph, kFaultDrainWait, nullptr);
                }
            }
        } else if ((warp == 9 || warp == 10) && lane == 0 && leader) {
            // ---------------- MMA issuers (even CTA): warp 9 tile 0, warp 10 tile 1 ----------------
            // One issuing thread per tile: each waits only on its own tile's barriers, so
            // while one waits (a wait costs the issuing thread 100-250 cycles even when the
            // barrier has completed, and only a few MMAs queue behind an issue) the other
            // keeps the tensor pipe fed. Both streams are shared-memory/K-major MMAs, so
            // their interleaving costs nothing. K/V slots and Q are released by both
            // issuers (barrier counts 2); a load that this tile does not read is released
            // only after it has landed, which puts the release in the slot's current phase.
            const int g = warp == 9 ? 0 : 1;
            auto kv_addr = [&](int s) { return base + kKvOff + static_cast<uint32_t>(s) * kSlotBytes; };
            auto issue_s = [&](uint32_t k_addr) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_f16_ss<2>(tmem + 128u * g, kmajor_desc(base + kQOff + g * kTileBytes, kk, 16384),
                                  kmajor_desc(k_addr, kk, 8192), kIdesc, kk > 0 ? 1u : 0u);
                mma_commit_pair(s_full(g), 0x3);
            };
            auto issue_pv = [&](uint32_t vt_addr, bool first) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_f16_ss<2>(tmem + 256u + 128u * g, kmajor_desc(base + kPOff + g * kTileBytes, kk, 16384),
                                  kmajor_desc(vt_addr, kk, 8192), kIdesc, (!first || kk > 0) ? 1u : 0u);
                mma_commit_pair(pv_done(g), 0x3);
            };
            int s_issued = 0, pv_issued = 0, outputs = 0;
            int kv_base = 0, items = 0;
            bool ok = true;
            // S_g may be overwritten once both CTAs' softmax warps hold its last block in registers.
            auto s_writable = [&]() {
                return s_issued == 0 ||
                       mbar_wait(s_free(g), static_cast<uint32_t>(s_issued - 1) & 1u, kFaultAttnWait, abort_flag);
            };
            for (int w = cluster_id; w < p.num_items && ok; w += num_clusters, ++items) {
                const PairItem it = make_pair_item(w, p);
                const int nb = it.nb[g];
                auto slot_of = [&](int load) { return (kv_base + load) % kSlots; };
                auto phase_of = [&](int load) { return static_cast<uint32_t>((kv_base + load) / kSlots) & 1u; };
                auto release_unused = [&](int load) {
                    if (!mbar_wait(kv_full(slot_of(load)), phase_of(load), kFaultAttnWait, abort_flag)) return false;
                    mma_commit_pair(kv_empty(slot_of(load)), 0x3);
                    return true;
                };
                // Q of this item has landed: q_empty is in this item's phase.
                ok = mbar_wait(q_full, static_cast<uint32_t>(items) & 1u, kFaultAttnWait, abort_flag);
                if (ok && nb == 0) {
                    for (int load = 0; load < 2 * it.nb_load && ok; ++load) ok = release_unused(load);
                    if (ok) mma_commit_pair(q_empty, 0x3);
                    kv_base += 2 * it.nb_load;
                    continue;
                }
                ok = ok && mbar_wait(kv_full(slot_of(0)), phase_of(0), kFaultAttnWait, abort_flag) && s_writable();
                if (!ok) break;
                tc_fence_after();
                issue_s(kv_addr(slot_of(0)));
                ++s_issued;
                mma_commit_pair(kv_empty(slot_of(0)), 0x3);
                if (nb == 1) mma_commit_pair(q_empty, 0x3);
                for (int j = 0; j < it.nb_load && ok; ++j) {
                    ok = false;
                    // S of block j + 1: runs while the softmax of block j does.
                    if (j + 1 < it.nb_load) {
                        const int k_load = 2 * (j + 1);
                        if (j + 1 < nb) {
                            if (!mbar_wait(kv_full(slot_of(k_load)), phase_of(k_load), kFaultAttnWait, abort_flag) ||
                                !s_writable())
                                break;
                            tc_fence_after();
                            issue_s(kv_addr(slot_of(k_load)));
                            ++s_issued;
                            mma_commit_pair(kv_empty(slot_of(k_load)), 0x3);
                            if (j + 1 == nb - 1) mma_commit_pair(q_empty, 0x3);
                        } else if (!release_unused(k_load)) {
                            break;
                        }
                    }
                    // PV of block j.
                    const int v_load = 2 * j + 1;
                    if (j < nb) {
                        if (!mbar_wait(kv_full(slot_of(v_load)), phase_of(v_load), kFaultAttnWait, abort_flag) ||
                            !mbar_wait(p_ready(g), static_cast<uint32_t>(pv_issued) & 1u, kFaultAttnWait, abort_flag))
                            break;
                        // The first PV of an item overwrites O_g: the previous item's O_g must
                        // have been read out of tensor memory by both CTAs.
                        if (j == 0 && outputs > 0 &&
                            !mbar_wait(o_empty(g), static_cast<uint32_t>(outputs - 1) & 1u, kFaultAttnWait, abort_flag))
                            break;
                        tc_fence_after();
                        issue_pv(kv_addr(slot_of(v_load)), j == 0);
                        ++pv_issued;
                        mma_commit_pair(kv_empty(slot_of(v_load)), 0x3);
                    } else if (!release_unused(v_load)) {
                        break;
                    }
                    ok = true;
                }
                ++outputs;
                kv_base += 2 * it.nb_load;
            }
        }
        __syncwarp();
    } else {
        setmaxnreg_inc<kRegsSoftmax>();
        // ---------------- softmax warpgroups (warps 0-3: tile 0, 4-7: tile 1) ----------------
        const int g = static_cast<int>(warp >> 2);
        const uint32_t quarter = warp & 3u;
        const int row = static_cast<int>(quarter * 32 + lane);
        const uint32_t lane_bits = (quarter * 32u) << 16;
        const uint32_t s_addr = tmem + lane_bits + 128u * g;
        const uint32_t o_addr = tmem + lane_bits + 256u + 128u * g;
        // This thread's P row in shared memory; plain stores (no asm), so the compiler can
        // interleave them with the exponentials. fence.proxy.async orders them before the
        // MMAs read P.
        uint8_t* const p_row = smem + kPOff + g * kTileBytes + row * 128;
        const uint32_t swz = static_cast<uint32_t>(row & 7);
        const uint32_t s_free_lead = mapa_shared(s_free(g), 0);
        const uint32_t p_ready_lead = mapa_shared(p_ready(g), 0);
        const uint32_t o_empty_lead = mapa_shared(o_empty(g), 0);
        const float c = p.scale_log2;
        uint32_t s_seen = 0;  // S_g completions consumed
        uint32_t pv_count = 0;  // PV_g MMAs announced (one per processed block)
        uint32_t turns = 0;     // blocks shared with the other tile processed so far
        bool ok = true;
        for (int w = cluster_id; w < p.num_items && ok; w += num_clusters) {
            const PairItem it = make_pair_item(w, p);
            const int nb = it.nb[g];
            if (nb == 0) continue;
            const int q_row = it.q0 + 256 * g + 128 * static_cast<int>(rank) + row;
            float m_run = -INFINITY;  // running reference point, log2 units
            float l_run = 0.0f;       // running sum of 2^(s c - m_run)
            for (int j = 0; j < nb; ++j) {
                if (!mbar_wait_warp(s_full(g), s_seen & 1u, kFaultAttnWait, abort_flag)) {
                    ok = false;
                    break;
                }
                ++s_seen;
                tc_fence_after();
                uint32_t r[128];
                load_row128(s_addr, r);
                // S_g is in registers: the next block's S may overwrite it.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(s_free_lead);
                const int kv0 = 128 * j;
                int limit = p.seq - kv0;
                if (p.causal) limit = min(limit, q_row - kv0 + 1);
                if (__any_sync(0xffffffffu, limit < 128)) mask_row128(r, limit);
                float m_use, alpha;
                next_point(m_run, row_max128(r) * c, m_use, alpha);
                // PV_g,j-1 must have completed before O_g is rescaled or P_g overwritten
                // (block 0's predecessor was waited for by the previous item's epilogue).
                if (j > 0 && !mbar_wait_warp(pv_done(g), (pv_count - 1) & 1u, kFaultAttnWait, abort_flag)) {
                    ok = false;
                    break;
                }
                bool rescaled = false;
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                    tc_fence_after();
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        uint32_t o[16];
                        tmem_ld_32x32b_x16(o_addr + 16 * cc, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st_32x32b_x16(o_addr + 16 * cc, o);
                    }
                    rescaled = true;
                }
                // Blocks that both tiles process take turns on the MUFU unit: tile 0's
                // exponentials of a shared block, then tile 1's, then tile 0's next, so the
                // other warp's loads, maximum and stores overlap them instead of competing.
                const bool shared_block = kMufuTurns && j < it.nb[0] && j < it.nb[1];
                if (shared_block && !(g == 0 && turns == 0) &&
                    !mbar_wait_warp(turn(g, quarter), static_cast<uint32_t>(g == 0 ? turns - 1 : turns) & 1u,
                                    kFaultAttnWait, abort_flag)) {
                    ok = false;
                    break;
                }
                // Exponentials (packed FP32 arguments and sums) and binary16 P, stored chunk by
                // chunk into the K-major 128-byte-swizzled tile: 16-byte chunk q of key box b at
                // row * 128 + ((q ^ (row % 8)) * 16).
                float2 acc[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) acc[t] = make_float2(0.0f, 0.0f);
                const float2 c2 = make_float2(c, c);
                const float2 m2 = make_float2(-m_use, -m_use);
#pragma unroll
                for (int ch = 0; ch < 16; ++ch) {
                    uint32_t pk[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int k2 = 8 * ch + 2 * i;
                        const float2 a =
                            fma2(make_float2(__uint_as_float(r[k2]), __uint_as_float(r[k2 + 1])), c2, m2);
                        const float2 e = make_float2(ex2(a.x), ex2(a.y));
                        acc[i] = add2(acc[i], e);
                        pk[i] = pack_half2(e.x, e.y);
                    }
                    *reinterpret_cast<uint4*>(p_row + (ch >> 3) * 16384 + ((static_cast<uint32_t>(ch & 7) ^ swz) << 4)) =
                        make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                if (shared_block) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(turn(1 - g, quarter));
                    ++turns;
                }
                const float2 s01 = add2(acc[0], acc[1]);
                const float2 s23 = add2(acc[2], acc[3]);
                const float2 st = add2(s01, s23);
                const float e_sum = st.x + st.y;
                fence_proxy_async_smem();
                if (rescaled) tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(p_ready_lead);
                ++pv_count;
                l_run = l_run * alpha + e_sum;
                m_run = m_use;
            }
            if (!ok || !mbar_wait_warp(pv_done(g), (pv_count - 1) & 1u, kFaultAttnWait, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const bool row_ok = q_row < p.seq;
            // One reciprocal of the row sum, then products (within 2^-23 relative of a
            // division, far inside the error bound).
            const float inv_l = __frcp_rn(l_run);
            float* orow = p.out + (static_cast<long long>(it.bh) * p.seq + q_row) * 128;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(o_addr + 32 * cc, o);
                tmem_wait_ld();
                if (cc == 3) {
                    // O_g is in registers: the next item's first PV may overwrite it.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(o_empty_lead);
                }
                if (row_ok) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        float4 v;
                        v.x = __uint_as_float(o[4 * q]) * inv_l;
                        v.y = __uint_as_float(o[4 * q + 1]) * inv_l;
                        v.z = __uint_as_float(o[4 * q + 2]) * inv_l;
                        v.w = __uint_as_float(o[4 * q + 3]) * inv_l;
                        float* dst = orow + 32 * cc + 4 * q;
                        if (p.out_vec4) {
                            __stcs(reinterpret_cast<float4*>(dst), v);
                        } else {
                            dst[0] = v.x;
                            dst[1] = v.y;
                            dst[2] = v.z;
                            dst[3] = v.w;
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the pair's MMAs may still read its shared memory
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc<2>(tmem, 512);
    }
}

// V [bh_kv, S, 128] -> V^T [bh_kv, 128, s_pad] (binary16), keys S..s_pad-1 zero.
// One 256-thread block per (64-key block, slice). Loads: a warp reads two whole
// 256-byte key rows (16-byte chunks, coalesced). Each thread packs the same head-dim
// column of two keys into one 32-bit word, so the shared tile holds key pairs,
// [128 head-dim rows][32 key pairs + 1]: the odd row pitch spreads a warp's
// transposing stores over 8 banks per key pair (at most 4 lanes per bank) and makes
// the reads of 4 consecutive key pairs conflict-free. Stores: 16-byte chunks of 8
// keys, 8 lanes per 128-byte V^T row segment.
__global__ void __launch_bounds__(256) transpose_v_kernel(const uint16_t* __restrict__ v, uint16_t* __restrict__ vt,
                                                          int seq, int s_pad, int slices) {
    __shared__ uint32_t tile[128][33];
    const int k0 = static_cast<int>(blockIdx.x) * 64;
    const int t = static_cast<int>(threadIdx.x);
    for (int slice = static_cast<int>(blockIdx.y); slice < slices; slice += static_cast<int>(gridDim.y)) {
        const uint16_t* src = v + static_cast<long long>(slice) * seq * 128LL;
        uint16_t* dst = vt + static_cast<long long>(slice) * 128LL * s_pad;
        __syncthreads();  // the previous slice's tile has been stored
        // 32 key pairs x 16 head-dim chunks of 8 = 512 units, two per thread.
        for (int u = t; u < 512; u += 256) {
            const int dc = u & 15;   // head-dim chunk: columns 8 dc .. 8 dc + 7
            const int kp = u >> 4;   // key pair: keys k0 + 2 kp, k0 + 2 kp + 1
            const int key = k0 + 2 * kp;
            uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
            if (key < seq) lo = *reinterpret_cast<const uint4*>(src + static_cast<long long>(key) * 128 + 8 * dc);
            if (key + 1 < seq) hi = *reinterpret_cast<const uint4*>(src + static_cast<long long>(key + 1) * 128 + 8 * dc);
            const uint32_t a[4] = {lo.x, lo.y, lo.z, lo.w};
            const uint32_t b[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                // columns 8 dc + 2 w (low halves) and 8 dc + 2 w + 1 (high halves)
                tile[8 * dc + 2 * w][kp] = (a[w] & 0xffffu) | (b[w] << 16);
                tile[8 * dc + 2 * w + 1][kp] = (a[w] >> 16) | (b[w] & 0xffff0000u);
            }
        }
        __syncthreads();
        // 128 head-dim rows x 8 chunks of 8 keys = 1024 units, four per thread.
        for (int u = t; u < 1024; u += 256) {
            const int d = u >> 3;
            const int kc = u & 7;  // keys k0 + 8 kc .. k0 + 8 kc + 7 = key pairs 4 kc .. 4 kc + 3
            const uint4 out = make_uint4(tile[d][4 * kc], tile[d][4 * kc + 1], tile[d][4 * kc + 2], tile[d][4 * kc + 3]);
            *reinterpret_cast<uint4*>(dst + static_cast<long long>(d) * s_pad + k0 + 8 * kc) = out;
        }
    }
}

// Host side: V^T into stream-ordered scratch, then the pair kernel on
// min(items, SMs / 2) clusters of two CTAs. q, k, v are 16-byte aligned.
inline cudaError_t launch(const void* q, const void* k, const void* v, float* out, int bh, int heads_q,
                          int heads_kv, int seq, float scale, int causal, int device, int sm_count,
                          cudaStream_t stream) {
    static std::atomic<bool> configured[host::kMaxDevices];
    if (!configured[device].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(attention_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBytes);
        if (e != cudaSuccess) return e;
        configured[device].store(true, std::memory_order_release);
    }
    PairParams p{};
    p.seq = seq;
    p.bh = bh;
    p.heads_q = heads_q;
    p.group = heads_q / heads_kv;
    p.heads_kv = heads_kv;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.causal = causal;
    p.out = out;
    p.out_vec4 = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    p.quads = (seq + kRowsPerItem - 1) / kRowsPerItem;
    p.num_items = bh * p.quads;
    const int bh_kv = bh / p.group;
    const int s_pad = (seq + 127) / 128 * 128;

    void* vt = nullptr;
    cudaError_t err = host::scratch_alloc(&vt, static_cast<size_t>(bh_kv) * 128 * s_pad * 2, device, stream);
    if (err != cudaSuccess) return err;
    const dim3 tgrid(static_cast<unsigned>(s_pad / 64), static_cast<unsigned>(bh_kv < 65535 ? bh_kv : 65535));
    transpose_v_kernel<<<tgrid, 256, 0, stream>>>(static_cast<const uint16_t*>(v), static_cast<uint16_t*>(vt), seq,
                                                  s_pad, bh_kv);
    CUtensorMap mq, mk, mvt;
    const uint64_t dq[3] = {128, static_cast<uint64_t>(seq), static_cast<uint64_t>(bh)};
    const uint64_t dk[3] = {128, static_cast<uint64_t>(seq), static_cast<uint64_t>(bh_kv)};
    const uint64_t sqk[2] = {256, 256ull * static_cast<uint64_t>(seq)};
    const uint64_t dvt[3] = {static_cast<uint64_t>(s_pad), 128, static_cast<uint64_t>(bh_kv)};
    const uint64_t svt[2] = {2ull * static_cast<uint64_t>(s_pad), 256ull * static_cast<uint64_t>(s_pad)};
    const uint32_t box_q[3] = {64, 128, 1};
    const uint32_t box_kv[3] = {64, 64, 1};
    if (!host::make_map_f16(&mq, q, 3, dq, sqk, box_q) || !host::make_map_f16(&mk, k, 3, dk, sqk, box_kv) ||
        !host::make_map_f16(&mvt, vt, 3, dvt, svt, box_kv)) {
        cudaFreeAsync(vt, stream);
        return cudaErrorInvalidValue;
    }
    const int clusters = p.num_items < sm_count / 2 ? p.num_items : sm_count / 2;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    err = cudaLaunchKernelEx(&cfg, attention_pair_kernel, mq, mk, mvt, p);
    cudaFreeAsync(vt, stream);
    return err;
}

}  // namespace pair
}  // namespace attn
}  // namespace tk
