/*
 * tk_b200.h — C ABI of the B200 (sm_100a) implementation of the
 * ThunderKittens-SM7x hot path.
 *
 * Plain C: pointers, sizes, a CUDA stream and a cudaError_t result. Binary16
 * (FP16) buffers are passed as `const void*` holding IEEE binary16 elements.
 * Reference citations are relative to the ThunderKittens-SM7x project root.
 *
 * Common contract (from include/tk_sm7x/gemm.cuh:8-14 and attention.cuh:8-14):
 *   - All pointers are device-accessible on the current device. The caller owns
 *     every buffer and keeps it alive until the stream work completes.
 *   - Work is enqueued asynchronously on `stream` (0 = legacy default stream;
 *     any stream, including non-blocking ones, is accepted).
 *   - Invalid arguments return cudaErrorInvalidValue before anything is
 *     enqueued: outputs are untouched and the thread's pending CUDA error is left
 *     as it was (src/gemm.cu:190-195, src/attention.cu:66-68).
 *   - A valid call first clears the pending error, enqueues, and returns
 *     cudaGetLastError() (src/gemm.cu:197-205). Success covers validation and
 *     launch only; execution errors surface at synchronisation.
 *   - A device without compute capability 10.0 returns
 *     cudaErrorInvalidDeviceFunction (the library holds sm_100a code only).
 */
#ifndef TK_B200_H
#define TK_B200_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TK_API __attribute__((visibility("default")))
#else
#define TK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- GEMM ------------------------------------------------------------------ */

/* Replaces tk_sm7x::gemm_f16_f16_f32_nn (include/tk_sm7x/gemm.cuh:15-20,
 * src/gemm.cu:184-206). C[m x n] = A[m x k] * B[k x n]; A, B row-major binary16,
 * C row-major FP32 with FP32 accumulation. m, n, k positive multiples of 16;
 * lda >= k, ldb >= n, ldc >= n; A, B, C must not overlap. Only the logical
 * m x n cells of C are written: columns n..ldc-1 of each row are untouched.
 * Any element alignment of the pointers and any leading dimension satisfying
 * the rule above is accepted (16-byte aligned rows take the TMA path directly;
 * other operands are first copied into stream-ordered scratch buffers). */
TK_API cudaError_t tk_gemm_f16_f16_f32_nn(int m, int n, int k, const void* a, int lda,
                                          const void* b, int ldb, float* c, int ldc,
                                          cudaStream_t stream);

/* GEMM with a fused row-statistics epilogue: in addition to C, row_max[i] and
 * row_sum[i] receive the maximum and sum of row i of the FP32 result C. The
 * reduction order is fixed: each 16-column group is reduced by the canonical
 * balanced tree (tests/row_reduce_reference.cuh:16-24), then groups combine
 * pairwise level by level in column order, an odd last partial carried up.
 * Max ties pick the right operand (include/tk_sm7x/row_reduce_ops.cuh:11-15).
 * Generalises examples/gemm_row_stats.cu:17-40 from one 16x16 tile to full rows.
 * row_max and row_sum hold m floats each and must not overlap C or each other.
 * The per-tile partials (m * ceil(n / 256) float pairs) live in a scratch
 * buffer taken stream-ordered (cudaMallocFromPoolAsync) from a memory pool the
 * library creates per device and returned with cudaFreeAsync on the same stream. */
TK_API cudaError_t tk_gemm_f16_f16_f32_nn_rowstats(int m, int n, int k, const void* a,
                                                   int lda, const void* b, int ldb,
                                                   float* c, int ldc, float* row_max,
                                                   float* row_sum, cudaStream_t stream);

/* Largest m * ceil(n / 256) accepted by tk_gemm_f16_f16_f32_nn_rowstats_noalloc:
 * the number of (max, sum) float pairs its built-in scratch holds (4 MiB). */
#define TK_GEMM_ROWSTATS_NOALLOC_MAX_PARTIALS (1u << 19)

/* No counterpart in the reference. The fused row-statistics GEMM above for
 * callers that must not allocate device memory: code that runs where cudaMalloc
 * and the stream-ordered allocator are off limits (a custom or arena allocator
 * that owns all device memory, a host process that forbids allocation after
 * start-up, or real-time paths where an allocation could block). It computes
 * exactly what tk_gemm_f16_f16_f32_nn_rowstats computes, but takes its per-tile
 * partials from a fixed 4 MiB array compiled into the library instead of
 * allocating them, and calls no allocation routine at all.
 *   - Limit: m * ceil(n / 256) must not exceed TK_GEMM_ROWSTATS_NOALLOC_MAX_PARTIALS
 *     (for example m = 8192 with n up to 16384); larger problems return
 *     cudaErrorNotSupported before anything is enqueued.
 *   - A and B must be TMA-addressable as given (16-byte aligned base pointers,
 *     lda and ldb multiples of 8); other layouts would need a repacking copy and
 *     return cudaErrorNotSupported. Other invalid arguments return
 *     cudaErrorInvalidValue, as for the other GEMM entry points.
 *   - The array lives on every GPU that loads the library until the process
 *     exits. The first call on a device looks up its device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before capturing the stream into a CUDA graph.
 *   - All calls share the array and each call overwrites the partials it uses
 *     before reading them. Calls whose kernels overlap on the GPU (different
 *     streams, or concurrent host threads on one device) race on it: order them
 *     on one stream or serialise them. */
TK_API cudaError_t tk_gemm_f16_f16_f32_nn_rowstats_noalloc(int m, int n, int k, const void* a,
                                                           int lda, const void* b, int ldb,
                                                           float* c, int ldc, float* row_max,
                                                           float* row_sum, cudaStream_t stream);

/* GEMM followed by a full-row softmax of its result, fused: C as
 * tk_gemm_f16_f16_f32_nn, and P[i][j] = exp(C[i][j] - max_j C[i]) / sum_j exp(...)
 * over each row's n columns. Generalises the reference's GEMM -> tile softmax
 * example (examples/gemm_row_softmax.cu:25-48) from one 16x16 tile to full rows. The GEMM
 * epilogue reduces each 256-column tile of a row to (tile max m_t, sum of
 * exp(C - m_t)) while the accumulator is still on chip; a second kernel merges the
 * pairs in tile order and writes P from C (one extra read of C). P is FP32
 * row-major with leading dimension ldp >= n. P may be C itself (probs == c and
 * ldp == ldc: C is replaced by P) or lie entirely outside C; A and B must not
 * overlap C or P. Accuracy: within 512 * 2^-23 of the FP64 softmax of the
 * returned C per element (the softmax bound of tests/tile_softmax.cu:20).
 * Scratch for the pairs (m * ceil(n / 256) float pairs) as for the row-statistics
 * entry point. */
TK_API cudaError_t tk_gemm_f16_f16_f32_nn_rowsoftmax(int m, int n, int k, const void* a,
                                                     int lda, const void* b, int ldb,
                                                     float* c, int ldc, float* probs, int ldp,
                                                     cudaStream_t stream);

/* Multi-GPU GEMM with the all-gather fused into the epilogue (no counterpart in
 * the reference, which has no multi-GPU code). Rank `rank` of `n_ranks`
 * (1 <= n_ranks <= 8) computes its m rows of C = A B and stores them, tile by
 * tile as the MMAs finish, at rows [rank * m, rank * m + m) of every rank's
 * gathered buffer c_ranks[0 .. n_ranks) (n_ranks * m rows, leading dimension
 * ldc): c_ranks[rank] is this rank's own buffer, the others are the peers'
 * buffers mapped into this process (tk_ipc_open), written over NVLink with plain
 * stores. A, B and the argument rules are those of tk_gemm_f16_f16_f32_nn. Rank r
 * may read its buffer once every rank's call has completed (the caller
 * synchronises its stream and then the ranks, e.g. with a host barrier). */
TK_API cudaError_t tk_gemm_f16_f16_f32_nn_gather(int m, int n, int k, const void* a, int lda,
                                                 const void* b, int ldb, float* const* c_ranks,
                                                 int n_ranks, int rank, int ldc,
                                                 cudaStream_t stream);

/* Device memory that other processes can map (for the gathered GEMM's buffers;
 * no counterpart in the reference). tk_ipc_alloc: cudaMalloc of `bytes` on the
 * current device and its cudaIpcMemHandle_t (64 bytes) in `handle`;
 * tk_ipc_open: maps a handle from another process (peer access enabled);
 * tk_ipc_close unmaps it; tk_ipc_free frees an allocation of tk_ipc_alloc. */
TK_API cudaError_t tk_ipc_alloc(size_t bytes, void** ptr, void* handle);
TK_API cudaError_t tk_ipc_open(const void* handle, void** ptr);
TK_API cudaError_t tk_ipc_close(void* ptr);
TK_API cudaError_t tk_ipc_free(void* ptr);

/* Tuning knob, no counterpart in the reference (whose tile choice is the fixed
 * rule of src/gemm.cu:50-57): 0 = choose by problem size (default), 1 = one CTA
 * per 128 x 256 tile, 2 = CTA pairs on 256 x 256 tiles. Process-wide; returns
 * the previous setting. */
TK_API int tk_gemm_set_cta_group(int cta_group);

/* Tuning knob, no counterpart in the reference: how split-K GEMMs (few output
 * tiles, long K) sum their K splits. 0 = inside the kernel, the splits of one
 * tile forming a thread-block cluster, whenever all tiles' clusters fit on the
 * GPU at once (default); 1 = always a second kernel over partials in scratch.
 * The split count does not depend on the mode and both add the splits in the
 * same order, so results are bit-identical. Process-wide; returns the previous
 * setting. */
TK_API int tk_gemm_set_splitk_reduce(int mode);

/* ---- tile row operations --------------------------------------------------- */
/* `tiles` holds n_tiles contiguous 16x16 row-major FP32 tiles (256 floats,
 * 1 KiB each). Reductions write 16 floats per tile (row order); softmax writes
 * 256 floats per tile. n_tiles == 0 is a valid empty call (nothing enqueued).
 * tiles and out must be 4-byte aligned; softmax outputs may alias the input
 * exactly (in place) but must not partially overlap it. */

/* Per-row sum, balanced column-order tree, replaces tk_sm7x::row_sum
 * (include/tk_sm7x/reduce.cuh:43-46) for a batch of tiles. */
TK_API cudaError_t tk_tile_row_sum_f32(const float* tiles, size_t n_tiles, float* out,
                                       cudaStream_t stream);
/* Per-row max, same tree, ties pick the right operand; replaces tk_sm7x::row_max
 * (include/tk_sm7x/reduce.cuh:48-51). */
TK_API cudaError_t tk_tile_row_max_f32(const float* tiles, size_t n_tiles, float* out,
                                       cudaStream_t stream);
/* exp(x - row_max) / row_sum with the same trees; replaces
 * tk_sm7x::row_softmax (include/tk_sm7x/softmax.cuh:54-64). */
TK_API cudaError_t tk_tile_row_softmax_f32(const float* tiles, size_t n_tiles,
                                           float* out, cudaStream_t stream);
/* Row i uses columns 0..i; the rest are exactly 0. Replaces
 * tk_sm7x::row_softmax_causal (include/tk_sm7x/softmax.cuh:69-81). */
TK_API cudaError_t tk_tile_row_softmax_causal_f32(const float* tiles, size_t n_tiles,
                                                  float* out, cudaStream_t stream);
/* All four from one read of the input. Any output may be NULL (skipped) but not
 * all of them; outputs must not overlap each other or the input. */
TK_API cudaError_t tk_tile_row_ops_f32(const float* tiles, size_t n_tiles,
                                       float* row_sum, float* row_max, float* softmax,
                                       float* softmax_causal, cudaStream_t stream);

/* ---- attention forward ------------------------------------------------------ */

/* Replace tk_sm7x::attention_forward_16x16[_causal] (include/tk_sm7x/
 * attention.cuh:15-23, src/attention.cu:76-86): softmax(Q K^T / 4) V for one
 * contiguous row-major 16x16 binary16 tile each of Q, K, V; the normalised
 * probabilities are rounded to binary16 (nearest even) before the PV product;
 * out is a contiguous row-major 16x16 FP32 tile. Q, K, V may alias each other
 * but not out. Inputs must be finite. */
TK_API cudaError_t tk_attention_forward_16x16(const void* q, const void* k,
                                              const void* v, float* out,
                                              cudaStream_t stream);
TK_API cudaError_t tk_attention_forward_16x16_causal(const void* q, const void* k,
                                                     const void* v, float* out,
                                                     cudaStream_t stream);

/* General forward over [batch, heads, seq, head_dim] contiguous binary16 Q, K, V
 * and FP32 out of the same shape: out = softmax(Q K^T * scale [causal: key t <=
 * query row]) V with the probabilities rounded to binary16 before the PV product.
 * head_dim in {16, 32, 64, 128}; seq >= 1 (tails allowed); batch, heads >= 1.
 * When seq <= 128 the probabilities are normalised before rounding (the exact
 * semantics of the 16x16 entry points); for longer sequences the kernel keeps a
 * running max and rounds exp(s - running_max) before the PV product, then
 * divides by the running sum (online softmax), which stays inside the
 * generalised error bound. Q, K, V may alias each other but not out. */
TK_API cudaError_t tk_attention_forward_f16(const void* q, const void* k, const void* v,
                                            float* out, int batch, int heads, int seq,
                                            int head_dim, float scale, int causal,
                                            cudaStream_t stream);

/* Grouped-query attention, a generalisation the reference rules out (README.md:35-36):
 * Q and out are [batch, heads_q, seq, head_dim], K and V are [batch, heads_kv,
 * seq, head_dim]; query head h attends with key/value head h / (heads_q /
 * heads_kv). heads_q must be a multiple of heads_kv; everything else as
 * tk_attention_forward_f16 (which is the heads_kv == heads_q case). */
TK_API cudaError_t tk_attention_forward_gqa_f16(const void* q, const void* k, const void* v,
                                                float* out, int batch, int heads_q, int heads_kv,
                                                int seq, int head_dim, float scale, int causal,
                                                cudaStream_t stream);

/* No counterpart in the reference (a tuning switch). GEMMs with m <= 64 (and no fused
 * epilogue) run on an operand-swapped kernel by default (1): C^T = B^T A^T, so the rows
 * of A become the tensor-core MMA's N dimension (16..64) and 128 columns of B its M;
 * 0 selects the 128-row tiles instead. Both are inside the same error bound. Returns
 * the previous setting; other values only query it. Process-wide. */
TK_API int tk_gemm_set_small_m(int mode);

/* No counterpart in the reference (a tuning switch). Tile-rows per rasterisation
 * group of the GEMM kernels' persistent tile walk: 0 (default) chooses by output shape
 * (16, or 32 when the output has at most 16 tile-columns); 1..4096 forces a value. The
 * walk decides which tiles sum their K-blocks in descending order (every other tile of
 * each CTA, when K is not split), so the last bits of C may change with it, inside the
 * same error bound. Returns the previous setting; other values only query it.
 * Process-wide; every call reads it. */
TK_API int tk_gemm_set_group_rows(int rows);

/* No counterpart in the reference (a tuning switch). Attention with head_dim 128,
 * more than 128 keys and a positive scale has two kernels: 1 (also 0, the
 * default) selects the single-CTA persistent kernel, 2 the CTA-pair kernel
 * (tcgen05 cta_group::2, M = 256 tiles, every MMA with both operands K-major in
 * shared memory). Both give results inside the same bound; the single-CTA kernel
 * is the faster on B200. Returns the previous setting (1 or 2); other values only
 * query it. Process-wide; every call reads it. */
TK_API int tk_attention_set_cta_group(int cta_group);

/* ---- status ------------------------------------------------------------------ */

/* Every wait inside the library's kernels is bounded. A kernel that gives up on
 * a wait records a nonzero code in a per-device status word and returns
 * instead of hanging; its outputs are then incomplete. This reads (and with
 * clear != 0 resets) that word for the current device; it synchronises the
 * device. While the word is nonzero, the finishing passes of the row-statistics
 * and row-softmax GEMMs write NaN instead of results built from per-tile
 * partials that a stopped GEMM may not have written. */
TK_API cudaError_t tk_device_status(uint32_t* status, int clear);

/* No counterpart in the reference (diagnostic). Bytes that the library's private
 * stream-ordered scratch pool on `device` has reserved from the driver
 * (*reserved) and currently hands out to allocations not yet freed (*used). The
 * pool is created by the first call on that device that needs scratch (repacked
 * operands, split-K partials, row-statistics pairs, the attention work counter);
 * until then both are 0. Device ordinal out of range: cudaErrorInvalidDevice. */
TK_API cudaError_t tk_scratch_pool_bytes(int device, uint64_t* reserved, uint64_t* used);

/* Version of this C ABI (major * 100 + minor). */
TK_API int tk_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TK_B200_H */
