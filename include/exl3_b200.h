/*
 * exl3_b200.h — C ABI of the B200 (sm_100a) routed-expert EXL3 MoE prefill library (libexl3_b200.so).
 *
 * Each entry point replaces one function of the reference's pybind/torch extensions; the reference
 * interface is cited beside it (paths within the reference project).  Conventions:
 *   - plain device pointers, sizes and element strides; fp16 data is passed as `const void*`;
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); every call is asynchronous on
 *     it and never synchronises the host;
 *   - calls launch on the CALLER's current CUDA device;
 *   - every call returns 0 on success or a non-zero error code; exl3_last_error() then returns a
 *     message for the calling thread (the torch shim raises it as RuntimeError, like the reference's
 *     TORCH_CHECK);
 *   - the caller allocates every buffer, outputs included (kernel/exl3_grouped_runtime.py:69-80);
 *     mode-1 / scatter outputs must be zeroed (or hold the values to accumulate onto) by the caller.
 *   - `status` (nullable) is a device int32 that a kernel sets to a non-zero EXL3_ERR_* code when it
 *     gives up (a bounded wait timed out, or routing ids out of range); the caller reads it whenever
 *     convenient.
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define EXL3_API __attribute__((visibility("default")))
#else
#define EXL3_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3_B200_ABI_VERSION 2

/* return codes */
#define EXL3_OK 0
#define EXL3_E_INVALID 1        /* invalid argument (shape, dtype code, alignment, size) */
#define EXL3_E_CUDA 2           /* a CUDA runtime call failed */

/* device status codes (written to `status`) */
#define EXL3_ERR_WAIT_TIMEOUT 1
#define EXL3_ERR_INVALID_EXPERT 2

/* weight dtype codes for exl3_route_sort */
#define EXL3_DTYPE_F32 0
#define EXL3_DTYPE_F16 1
#define EXL3_DTYPE_BF16 2

/* Message for the last failed call on this thread ("" if none). */
EXL3_API const char* exl3_last_error(void);

/* EXL3_B200_ABI_VERSION of the loaded library. */
EXL3_API int exl3_abi_version(void);

/* Time limit, in nanoseconds, of every bounded mbarrier wait in the tcgen05 kernels (grouped GEMM,
 * fat GEMM, router) launched after this call; process-wide.  A wait that runs past it makes the kernel
 * record EXL3_ERR_WAIT_TIMEOUT in `status`, stop every role, drain its copies and MMAs in flight, free
 * its tensor memory and return; its outputs are then incomplete.  ns < 0 restores the default (2 s).
 * Returns the previous limit.  No counterpart in the reference (its kernels have no timeouts); a
 * caller that needs a hang detector shorter than 2 s, and the tests of the timeout path, set it. */
EXL3_API int64_t exl3_set_wait_limit_ns(int64_t ns);

/* Stage 1a — per-expert M-block table.
 * Replaces build_blocks(counts, block_expert, block_row0, meta), kernel/exl3_grouped_prefill.cu:285-294
 * (kernel :63-96).  counts int32[n_experts] (n_experts <= 1024) -> block_expert/block_row0
 * int32[max_blocks], meta int32[2] = {n_blocks, n_rows}; entries past n_blocks get block_expert = -1
 * and keep their block_row0.  Bit-identical to the reference. */
EXL3_API int exl3_build_blocks(const int32_t* counts, int64_t n_experts, int32_t* block_expert, int32_t* block_row0,
                      int64_t max_blocks, int32_t* meta, void* stream);

/* Stage 1 (fused) — stable expert sort + block table, two launches, no host synchronisation.
 * Replaces the host sort block of grouped_prefill, kernel/exl3_grouped_runtime.py:59-72 (argsort
 * stable, token_sorted, weight_sorted, expert_of_row, counts, expert_row0, build_blocks).
 * scratch: device int32[scratch_elems], scratch_elems >= exl3_route_sort_scratch_elems(T*topk, n_experts)
 * (per-chunk expert histograms; contents on entry are ignored).
 * ids [T*topk] int64 (ids_is_int64 = 1) or int32; weights [T*topk] of weight_dtype.  Outputs:
 * token_sorted int64[R], weight_sorted fp16[R], expert_of_row int32[R], counts int32[n_experts],
 * expert_row0 int32[n_experts], block tables as exl3_build_blocks.  Bit-identical to the reference
 * for ids in [0, n_experts); other ids are not routed and counted in *invalid_count (device int32,
 * nullable). */
EXL3_API int exl3_route_sort(const void* ids, int ids_is_int64, const void* weights, int weight_dtype, int64_t T,
                    int64_t topk, int64_t n_experts, int64_t max_blocks, int64_t* token_sorted,
                    void* weight_sorted, int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0,
                    int32_t* block_expert, int32_t* block_row0, int32_t* meta, int32_t* invalid_count,
                    int32_t* scratch, int64_t scratch_elems, void* stream);

/* int32 elements of scratch exl3_route_sort needs for `rows` = T*topk routed rows (-1: bad arguments).
 * No counterpart in the reference (its sort ran as torch ops). */
EXL3_API int64_t exl3_route_sort_scratch_elems(int64_t rows, int64_t n_experts);

/* exl3_route_sort for callers that cannot allocate device memory while they run the prefill — an
 * engine that has already given nearly all of the GPU to its KV cache, or a host program driving this
 * C ABI without a device allocator of its own.  It takes no scratch argument and allocates nothing:
 * the chunk histograms live in a 256 KiB array inside the library (65536 int32), which every GPU that
 * loads the library keeps until the process exits.  Routings whose exl3_route_sort_scratch_elems()
 * exceeds 65536 (for example more than ~460K routed rows at 288 experts, ~129K at 1024) are rejected
 * with EXL3_E_INVALID.  The first call on a device, made with that device current, looks up the
 * array's device address; make that first call before any stream capture.  All calls share the one
 * array, so calls that overlap on the GPU (different streams or threads) race; serialise them.
 * Outputs and bit-exact results are those of exl3_route_sort.
 * No counterpart in the reference. */
EXL3_API int exl3_route_sort_noalloc(const void* ids, int ids_is_int64, const void* weights, int weight_dtype,
                                     int64_t T, int64_t topk, int64_t n_experts, int64_t max_blocks,
                                     int64_t* token_sorted, void* weight_sorted, int32_t* expert_of_row,
                                     int32_t* counts, int32_t* expert_row0, int32_t* block_expert,
                                     int32_t* block_row0, int32_t* meta, int32_t* invalid_count, void* stream);

/* Routing front-end (no reference kernel: the reference receives topk_ids / topk_weights from vLLM's
 * router).  GLM-5.3-Flash's router (docs/research/02-glm-5.3-flash-architecture.md:33): sigmoid scores
 * of x . w_router^T (fp32 accumulation of fp16 products), the topk experts by score + bias (noaux_tc
 * with one group), weights = score / (sum of the topk scores + 1e-20) if norm, times scale.
 * x fp16 [T, d], w_router fp16 [E, d] (the checkpoint's bf16 router weight converted once), bias fp32
 * [E] or NULL (zeros).  Outputs ids int64 [T, topk] (descending score + bias, ties to the lower id) and
 * weights fp32 [T, topk].  d % 64 == 0; 16 <= E <= 512, E % 16 == 0 and E splitting into equal
 * 16-multiples of at most 256 (288 = 2 x 144); topk <= 16.  One launch, 128 tokens per CTA. */
EXL3_API int exl3_router_topk(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E,
                              const float* bias, int64_t topk, int64_t norm, double scale, int64_t* ids,
                              float* weights, int32_t* status, void* stream);

/* int32 elements of scratch exl3_route_front needs (-1: bad arguments). */
EXL3_API int64_t exl3_route_front_scratch_elems(int64_t T, int64_t topk, int64_t E);

/* exl3_router_topk followed by the expert sort of exl3_route_sort over its output (same outputs and
 * bit-exact order as exl3_route_sort on those ids / weights).  When 2048 % (128 * topk) == 0 (topk 1, 2,
 * 4, 8, 16) the router kernel also produces the sort's chunk histograms, so the whole front-end is two
 * launches; otherwise three. */
EXL3_API int exl3_route_front(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E,
                              const float* bias, int64_t topk, int64_t norm, double scale, int64_t* ids,
                              float* weights, int64_t* token_sorted, void* weight_sorted, int32_t* expert_of_row,
                              int32_t* counts, int32_t* expert_row0, int32_t* block_expert, int32_t* block_row0,
                              int64_t max_blocks, int32_t* meta, int32_t* scratch, int64_t scratch_elems,
                              int32_t* status, void* stream);

/* exl3_route_front with token_sorted replaced by slot_sorted: the routing slot t*topk + j of every sorted
 * row (the sort of exl3_route_sort over the router's ids viewed as [T*topk, 1]), for the slot-ordered
 * down stage (exl3_grouped_gemm mode 2 + exl3_combine_slots).  No counterpart in the reference. */
EXL3_API int exl3_route_front_slots(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E,
                                   const float* bias, int64_t topk, int64_t norm, double scale, int64_t* ids,
                                   float* weights, int64_t* slot_sorted, void* weight_sorted, int32_t* expert_of_row,
                                   int32_t* counts, int32_t* expert_row0, int32_t* block_expert, int32_t* block_row0,
                                   int64_t max_blocks, int32_t* meta, int32_t* scratch, int64_t scratch_elems,
                                   int32_t* status, void* stream);

/* Stage 5b — per-token combine of the slot-ordered down rows.  y fp32 [T*topk, K] (row t*topk + j = route
 * j of token t, as exl3_grouped_gemm mode 2 stores it), ids [T, topk] int64 (ids_is_int64) or int32;
 * out fp32 [T, K] = (accumulate ? out : 0) + the sum over j ascending of the rows whose id is in
 * [0, n_experts) (fp32, deterministic; unrouted tokens get 0).  Replaces the atomic scatter of
 * grouped_gemm mode 1 (kernel/exl3_grouped_prefill.cu:274-275) in the single-GPU pipeline: same sum,
 * fixed order, no fp32 atomics.  topk <= 32, K % 128 == 0. */
EXL3_API int exl3_combine_slots(const float* y, const void* ids, int ids_is_int64, int64_t T, int64_t topk,
                               int64_t n_experts, float* out, int64_t K, int accumulate, void* stream);

/* Stage 2 — gather + input Hadamard.
 * Replaces row_had(src, dst, token_sorted, expert_of_row, suh, gather), kernel/exl3_grouped_prefill.cu:297-311.
 * dst fp16[rows, K] = H128( src[token_sorted[r] (gather) or r] (.) suh[expert_of_row[r]] ) / sqrt(128)
 * per 128-column block.  src fp16[src_rows, K]; suh fp16 rows of K with row stride suh_stride
 * (elements; the reference passes the strided view w13_suh[:, 0]).  K % 128 == 0. */
EXL3_API int exl3_row_had(const void* src, int64_t src_rows, void* dst, int64_t rows, int64_t K,
                 const int64_t* token_sorted, const int32_t* expert_of_row, const void* suh,
                 int64_t suh_stride, int gather, void* stream);

/* Stage 4 — clamped SwiGLU + down-projection input Hadamard.
 * Replaces act_had(gu, act, expert_of_row, suh_down, limit), kernel/exl3_grouped_prefill.cu:313-322.
 * gu fp16[rows, 2I] (gate | up) -> act fp16[rows, I]; I % 128 == 0. */
EXL3_API int exl3_act_had(const void* gu, void* act, int64_t rows, int64_t I, const int32_t* expert_of_row,
                 const void* suh_down, int64_t suh_stride, double limit, void* stream);

/* Stages 3 and 5 — grouped trellis GEMM over all experts (tcgen05 / TMEM).
 * Replaces grouped_gemm(a, packed_gate, packed_up, svh_gate, svh_up, block_expert, block_row0, counts,
 * expert_row0, token_sorted, route_weight, out, mode), kernel/exl3_grouped_prefill.cu:326-378.
 *   a            fp16 [rows, size_k] contiguous (sorted rows)
 *   packed_gate  int16 [n_experts, tiles_k, tiles_n, 64], inner dims contiguous, expert stride
 *                expert_stride_words (may exceed tiles_k*tiles_n*64: [E,2,...] views)
 *   packed_up    same layout and stride, or NULL (down stage)
 *   svh_gate/up  fp16 [n_experts, N] with row stride svh_stride (N = 16*tiles_n)
 *   block_expert, block_row0 (max_blocks entries): accepted for signature compatibility; the kernel
 *                schedules its own 256-row tiles from counts / expert_row0
 *   counts, expert_row0 int32 [n_experts]
 *   token_sorted int64 [rows], route_weight fp16 [rows] (mode 1)
 *   mode 0       out fp16 [rows, out_cols = 2N (or N without packed_up)]: gate | up
 *   mode 1       out fp32 [out_rows, out_cols = N] += route_weight[r] * y[r] at token_sorted[r]
 *                (atomic; order-nondeterministic like the reference).
 *   mode 2       out fp32 [out_rows, out_cols = N]: row token_sorted[r] = route_weight[r] * y[r], a plain
 *                row store (each destination row must be written by one sorted row).  No counterpart in
 *                the reference: with the routing sorted by slot (token_sorted holding t*topk + j, see
 *                exl3_route_sort over ids viewed as [T*topk, 1]) it writes every route's weighted row
 *                once, and exl3_combine_slots then sums each token's rows without atomics. */
EXL3_API int exl3_grouped_gemm(const void* a, int64_t rows, int64_t size_k, const int16_t* packed_gate,
                      const int16_t* packed_up, int64_t n_experts, int64_t tiles_k, int64_t tiles_n,
                      int64_t expert_stride_words, const void* svh_gate, const void* svh_up,
                      int64_t svh_stride, const int32_t* block_expert, const int32_t* block_row0,
                      int64_t max_blocks, const int32_t* counts, const int32_t* expert_row0,
                      const int64_t* token_sorted, const void* route_weight, void* out, int64_t out_rows,
                      int64_t out_cols, int64_t mode, int32_t* status, void* stream);

/* Per-expert trellis GEMM, direct store.
 * Replaces fat_gemm_v2(a, packed, out, svh, K, mcg, mul1, variant), kernel/exl3_fat_gemm_v2.cu:298-303.
 * a fp16 [size_m, size_k]; packed int16 [size_k/16, size_n/16, 64] contiguous; out fp32 [size_m, size_n];
 * svh fp16 [size_n].  K (bits) must be 4, mcg 1, mul1 0 (kernel/exl3_fat_gemm_v2.cu:246); variant 0..3
 * selects the reference's pipeline variant and is accepted for compatibility (one sm_100a kernel
 * serves all four). */
EXL3_API int exl3_fat_gemm_v2(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed, int64_t size_n,
                     float* out, const void* svh, int64_t K, int mcg, int mul1, int64_t variant,
                     int32_t* status, void* stream);

/* Per-expert trellis GEMM, route-weighted scatter: out[token_idx[r]] += route_weight[r] * y[r]
 * (non-atomic: one route per token per expert).
 * Replaces fat_gemm_v2_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1, variant),
 * kernel/exl3_fat_gemm_v2.cu:305-314.  out fp32 [out_rows, size_n]. */
EXL3_API int exl3_fat_gemm_v2_scatter(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed,
                             int64_t size_n, float* out, int64_t out_rows, const void* svh,
                             const int64_t* token_idx, const void* route_weight, int64_t K, int mcg,
                             int mul1, int64_t variant, int32_t* status, void* stream);

/* Dynamic shared memory of the kernel serving `variant` (0..3), -1 for an unknown variant.
 * Replaces smem_bytes(variant), kernel/exl3_fat_gemm_v2.cu:316-326. */
EXL3_API int64_t exl3_smem_bytes(int64_t variant);

/* PR77's original names (kernel/test_fat_v2.py:122 and :134): same as fat_gemm_v2 / _scatter with
 * variant 0. */
EXL3_API int exl3_fat_gemm(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed, int64_t size_n,
                  float* out, const void* svh, int64_t K, int mcg, int mul1, int32_t* status, void* stream);
EXL3_API int exl3_fat_gemm_scatter(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed,
                          int64_t size_n, float* out, int64_t out_rows, const void* svh,
                          const int64_t* token_idx, const void* route_weight, int64_t K, int mcg, int mul1,
                          int32_t* status, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Expert parallelism.  No reference counterpart: the reference refuses expert-parallel layers
 * (kernel/exl3_grouped_runtime.py:96-98, `layer.expert_map is not None` falls back).  One process per
 * GPU, at most 8.  Experts are placed E/N per rank: routing ids are expert POSITIONS (ids_pos, int64,
 * -1 = unrouted) and rank r owns positions [r*E/N, (r+1)*E/N).  Tokens live in per-rank blocks of
 * tokens_per_rank (tpr) rows: global token t is row t % tpr of rank t / tpr.  Every rank sorts the
 * all-gathered routing as one [N*tpr*topk] list (topk = 1 in exl3_route_sort), so a sorted row carries
 * its routing slot s = t*topk + j.
 *
 * Each rank publishes two buffers from exl3_ep_alloc, mapped by the others with exl3_ep_ipc_open: its
 * fp16 tokens [tpr, K] and a staging buffer [tpr * N, K] (fp16 or fp32) with one row per (token, source
 * rank).  Per layer:
 *   exl3_ep_pull_rows      each needed remote token row crosses NVLink once into a local [N*tpr, K] copy;
 *   exl3_ep_row_had        stage 2 gathers from it (own tokens from the own buffer), records slot_row;
 *   stages 3-4             exl3_grouped_gemm mode 0 and exl3_ep_act_had on the rank's experts;
 *   exl3_ep_gemm_store     stage 5 stores the weighted rows w[r] * y[r] locally;
 *   exl3_ep_combine_push   one summed row per (token, this rank) into the token owner's staging buffer;
 *   (barrier)              the caller's collective orders every rank's pushes before the reduce;
 *   exl3_ep_combine_reduce sums each token's rows over the contributing ranks in rank order.
 * The caller orders the ranks with two small collectives per layer (routing all-gather before the pull,
 * barrier before the reduce).
 * ------------------------------------------------------------------------------------------- */
#define EXL3_IPC_HANDLE_BYTES 64

/* cudaMalloc / cudaFree on the current device: the buffers whose IPC handles are shared. */
EXL3_API int exl3_ep_alloc(int64_t bytes, void** ptr);
EXL3_API int exl3_ep_free(void* ptr);
/* Export (64 bytes into `handle`) / map / unmap a buffer from exl3_ep_alloc of another process. */
EXL3_API int exl3_ep_ipc_handle(const void* ptr, void* handle);
EXL3_API int exl3_ep_ipc_open(const void* handle, void** ptr);
EXL3_API int exl3_ep_ipc_close(void* ptr);

/* Dispatch: x_pulled[t] = x_ranks[t / tpr][t % tpr] for every token t of ANOTHER rank with some
 * ids_pos[t*topk + j] in [e0, e1); other rows of x_pulled [n_ranks*tpr, K] fp16 are left untouched.
 * ids_pos [n_ranks*tpr, topk].  x_ranks is a HOST array of n_ranks device pointers.  No-op for 1 rank. */
EXL3_API int exl3_ep_pull_rows(const void* const* x_ranks, int64_t n_ranks, int64_t rank, int64_t tokens_per_rank,
                               int64_t K, const int64_t* ids_pos, int64_t topk, int64_t e0, int64_t e1,
                               void* x_pulled, void* stream);

/* Stage 2: dst[r] = H128(x(slot_sorted[r] / topk) (.) suh[expert_of_row[r] - expert_base]) where
 * x(t) = x_ranks[t / tpr][t % tpr] (x_ranks: HOST array of n_ranks device pointers; in the pipeline
 * above, the own token buffer for this rank and x_pulled + r*tpr*K for the others).  If slot_row is not
 * null, slot_row[slot_sorted[r]] = r ([n_ranks*tpr*topk] int32).  rows_dev (nullable): a device int32
 * row count (the sort's meta[1]); then min(rows, *rows_dev) rows are processed, `rows` being an upper
 * bound that sizes the grid, so no host read of the count is needed.  With n_ranks = 1 this is the
 * single-GPU row_had over a routing sorted by slot (token = slot / topk). */
EXL3_API int exl3_ep_row_had(const void* const* x_ranks, int64_t n_ranks, int64_t tokens_per_rank, int64_t topk,
                             void* dst, int64_t rows, int64_t K, const int64_t* slot_sorted,
                             const int32_t* expert_of_row, int64_t expert_base, const void* suh, int64_t suh_stride,
                             int32_t* slot_row, const int32_t* rows_dev, void* stream);

/* Stage 4 on a rank's expert slice: exl3_act_had with suh_down row expert_of_row[r] - expert_base, over
 * min(rows, *rows_dev) rows when rows_dev (a device int32 count) is given. */
EXL3_API int exl3_ep_act_had(const void* gu, void* act, int64_t rows, int64_t I, const int32_t* expert_of_row,
                             int64_t expert_base, const void* suh_down, int64_t suh_stride, double limit,
                             const int32_t* rows_dev, void* stream);

/* Stage 5: the down GEMM of exl3_grouped_gemm over this rank's experts, storing the weighted rows
 * y_local[r] = w[r] * y[r] (fp32 [rows, N], a caller workspace) instead of scattering them. */
EXL3_API int exl3_ep_gemm_store(const void* a, int64_t rows, int64_t size_k, const int16_t* packed,
                                int64_t n_experts, int64_t tiles_k, int64_t tiles_n, int64_t expert_stride_words,
                                const void* svh, int64_t svh_stride, const int32_t* counts,
                                const int32_t* expert_row0, const void* route_weight, float* y_local,
                                int32_t* status, void* stream);

/* Combine, expert side: for every token t in [0, n_ranks*tpr) with some ids_pos[t*topk + j] in [e0, e1),
 * staging_ranks[t / tpr] row (t % tpr) * n_ranks + rank = sum over those j, ascending, of
 * y_local[slot_row[t*topk + j]] (fp32 sum; stored fp16 if staging_f16 else fp32).  staging_ranks is a
 * HOST array of n_ranks device pointers. */
EXL3_API int exl3_ep_combine_push(const float* y_local, int64_t K, const int64_t* ids_pos, int64_t topk, int64_t e0,
                                  int64_t e1, const int32_t* slot_row, void* const* staging_ranks, int64_t n_ranks,
                                  int64_t rank, int64_t tokens_per_rank, int64_t staging_f16, void* stream);

/* Combine, owner side: out[t] = sum, over the ranks r (ascending) owning any ids_pos[t*topk + j] in
 * [0, n_experts), of staging[t * n_ranks + r] (fp32 accumulation; zeros for unrouted tokens).
 * staging [T * n_ranks, K] this rank's (fp16 if staging_f16 else fp32), ids_pos [T, topk], out fp32 [T, K]. */
EXL3_API int exl3_ep_combine_reduce(const void* staging, int64_t staging_f16, const int64_t* ids_pos, int64_t T,
                                    int64_t topk, int64_t n_experts, int64_t n_ranks, float* out, int64_t K,
                                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_B200_H */
