// route.cu — expert sort and per-expert M-block table (stage 1 of the grouped prefill).
//
// route_sort_kernel replaces the host-side torch sequence of kernel/exl3_grouped_runtime.py:59-67
// (stable argsort by expert, token/weight/expert arrays, bincount, exclusive cumsum) AND the
// build_blocks launch of :72 with ONE single-CTA kernel.  Results are bit-identical to the
// reference: the sort is a stable counting sort whose per-warp segments are ranked in order
// (__match_any_sync groups, lane order within a batch, warp order across segments).
//
// build_blocks_kernel keeps the reference's own entry point (kernel/exl3_grouped_prefill.cu:63-96,
// host fn :285-294) with the serial scan replaced by a block-wide parallel scan.
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "exl3_internal.h"

namespace exl3b {

namespace {

constexpr int ROUTE_THREADS = 1024;
constexpr int ROUTE_WARPS = ROUTE_THREADS / 32;
constexpr int ROUTE_UNROLL = 8;   // batches of 32 ids loaded ahead per warp

// Exclusive block-wide scan of one int per thread (1024 threads).  Returns the exclusive prefix and
// writes the block total to *total (visible to all threads on return).
__device__ __forceinline__ int block_scan_excl(int v, int* s_warp, int* total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1)
    {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0)
    {
        int w = s_warp[lane];
        int incl = w;
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1)
        {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        s_warp[lane] = incl - w;                 // exclusive prefix of warp totals
        if (lane == 31) *total = incl;
    }
    __syncthreads();
    const int r = s_warp[warp] + x - v;
    __syncthreads();                             // s_warp may be reused by the caller's next scan
    return r;
}

__device__ __forceinline__ int64_t load_id(const void* ids, int ids_i64, int64_t i)
{
    return ids_i64 ? __ldg(reinterpret_cast<const long long*>(ids) + i)
                   : (int64_t) __ldg(reinterpret_cast<const int*>(ids) + i);
}

__device__ __forceinline__ __half load_weight_f16(const void* w, int wdtype, int64_t i)
{
    if (wdtype == 0) return __float2half_rn(__ldg(reinterpret_cast<const float*>(w) + i));
    if (wdtype == 1) return reinterpret_cast<const __half*>(w)[i];
    return __float2half_rn(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]));
}

// Block table from per-expert counts held by thread e (< n_experts) in `c`.  Shared by both kernels.
__device__ __forceinline__ void write_block_table(int c, int n_experts, int max_blocks, int32_t* block_expert,
                                                  int32_t* block_row0, int32_t* meta, int* s_warp, int* s_tot)
{
    const int e = threadIdx.x;
    const int nblk = (e < n_experts) ? (c + 127) / 128 : 0;
    const int row0 = block_scan_excl(e < n_experts ? c : 0, s_warp, &s_tot[0]);
    const int blk0 = block_scan_excl(nblk, s_warp, &s_tot[1]);
    const int nb = s_tot[1];
    if (e < n_experts)
        for (int i = 0; i < nblk; ++i)
        {
            const int b = blk0 + i;
            if (b < max_blocks) { block_expert[b] = e; block_row0[b] = row0 + i * 128; }
        }
    for (int b = nb + e; b < max_blocks; b += ROUTE_THREADS) block_expert[b] = -1;
    if (e == 0) { meta[0] = nb; meta[1] = s_tot[0]; }
}

__global__ __launch_bounds__(ROUTE_THREADS, 1)
void route_sort_kernel(const void* __restrict__ ids, int ids_i64, const void* __restrict__ weights, int wdtype,
                       int64_t R, int topk, int n_experts, int max_blocks,
                       int64_t* __restrict__ token_sorted, __half* __restrict__ weight_sorted,
                       int32_t* __restrict__ expert_of_row, int32_t* __restrict__ counts,
                       int32_t* __restrict__ expert_row0, int32_t* __restrict__ block_expert,
                       int32_t* __restrict__ block_row0, int32_t* __restrict__ meta,
                       int32_t* __restrict__ invalid_count)
{
    extern __shared__ int32_t hist[];        // [ROUTE_WARPS][n_experts]: per-warp counts, then bases
    __shared__ int s_warp[32];
    __shared__ int s_tot[2];
    __shared__ int s_invalid;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int E = n_experts;

    for (int i = t; i < ROUTE_WARPS * E; i += ROUTE_THREADS) hist[i] = 0;
    if (t == 0) s_invalid = 0;
    __syncthreads();

    // Each warp owns one contiguous segment of the flattened ids, a whole number of 32-id batches.
    const int64_t nbatch = (R + 31) / 32;
    const int64_t per_warp = (nbatch + ROUTE_WARPS - 1) / ROUTE_WARPS;
    const int64_t b_lo = warp * per_warp;
    const int64_t b_hi = min(nbatch, b_lo + per_warp);
    int32_t* my_hist = hist + warp * E;

    // ---- pass 1: per-warp histograms
    for (int64_t b0 = b_lo; b0 < b_hi; b0 += ROUTE_UNROLL)
    {
        int key[ROUTE_UNROLL];
        #pragma unroll
        for (int u = 0; u < ROUTE_UNROLL; ++u)
        {
            const int64_t i = (b0 + u) * 32 + lane;
            key[u] = -2;                                           // -2: past the end
            if (b0 + u < b_hi && i < R)
            {
                const int64_t e = load_id(ids, ids_i64, i);
                key[u] = (e >= 0 && e < E) ? (int) e : -1;         // -1: not routed (invalid id)
            }
        }
        #pragma unroll
        for (int u = 0; u < ROUTE_UNROLL; ++u)
        {
            if (b0 + u >= b_hi) break;
            const unsigned peers = __match_any_sync(0xffffffffu, key[u]);
            if (key[u] == -1 && lane == __ffs(peers) - 1) atomicAdd(&s_invalid, __popc(peers));
            if (key[u] >= 0 && lane == __ffs(peers) - 1) my_hist[key[u]] += __popc(peers);
            __syncwarp();
        }
    }
    __syncthreads();

    // ---- scans: per expert over warps, then over experts
    int c = 0;
    if (t < E)
    {
        int run = 0;
        for (int w = 0; w < ROUTE_WARPS; ++w)
        {
            const int v = hist[w * E + t];
            hist[w * E + t] = run;
            run += v;
        }
        c = run;
    }
    const int row0 = block_scan_excl(t < E ? c : 0, s_warp, &s_tot[0]);
    if (t < E)
    {
        counts[t] = c;
        expert_row0[t] = row0;
        for (int w = 0; w < ROUTE_WARPS; ++w) hist[w * E + t] += row0;
    }
    __syncthreads();

    // ---- pass 2: stable scatter
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int64_t b0 = b_lo; b0 < b_hi; b0 += ROUTE_UNROLL)
    {
        int key[ROUTE_UNROLL];
        __half wv[ROUTE_UNROLL];
        #pragma unroll
        for (int u = 0; u < ROUTE_UNROLL; ++u)
        {
            const int64_t i = (b0 + u) * 32 + lane;
            key[u] = -2;
            wv[u] = __float2half(0.0f);
            if (b0 + u < b_hi && i < R)
            {
                const int64_t e = load_id(ids, ids_i64, i);
                key[u] = (e >= 0 && e < E) ? (int) e : -1;
                wv[u] = load_weight_f16(weights, wdtype, i);
            }
        }
        #pragma unroll
        for (int u = 0; u < ROUTE_UNROLL; ++u)
        {
            if (b0 + u >= b_hi) break;
            const unsigned peers = __match_any_sync(0xffffffffu, key[u]);
            int pos = 0;
            if (key[u] >= 0) pos = my_hist[key[u]] + __popc(peers & lt_mask);
            __syncwarp();
            if (key[u] >= 0 && lane == __ffs(peers) - 1) my_hist[key[u]] += __popc(peers);
            __syncwarp();
            if (key[u] >= 0)
            {
                const int64_t i = (b0 + u) * 32 + lane;
                token_sorted[pos] = i / topk;
                weight_sorted[pos] = wv[u];
                expert_of_row[pos] = key[u];
            }
        }
    }

    // ---- rows left over by ids outside [0, E) (only when some were invalid): token 0, expert 0,
    // weight 0, so that the row-wise stages that run over all R rows stay in bounds.
    for (int64_t i = (int64_t) s_tot[0] + t; i < R; i += ROUTE_THREADS)
    {
        token_sorted[i] = 0;
        weight_sorted[i] = __float2half(0.0f);
        expert_of_row[i] = 0;
    }

    // ---- block table (same semantics as build_blocks)
    write_block_table(c, E, max_blocks, block_expert, block_row0, meta, s_warp, s_tot);
    if (t == 0 && invalid_count) *invalid_count = s_invalid;
}

__global__ __launch_bounds__(ROUTE_THREADS, 1)
void build_blocks_kernel(const int32_t* __restrict__ counts, int n_experts, int max_blocks,
                         int32_t* __restrict__ block_expert, int32_t* __restrict__ block_row0,
                         int32_t* __restrict__ meta)
{
    __shared__ int s_warp[32];
    __shared__ int s_tot[2];
    const int e = threadIdx.x;
    const int c = (e < n_experts) ? counts[e] : 0;
    write_block_table(c, n_experts, max_blocks, block_expert, block_row0, meta, s_warp, s_tot);
}

}  // namespace

int launch_route_sort(const void* ids, int ids_i64, const void* weights, int wdtype, int64_t T, int topk,
                      int n_experts, int max_blocks, int64_t* token_sorted, void* weight_sorted,
                      int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0, int32_t* block_expert,
                      int32_t* block_row0, int32_t* meta, int32_t* invalid_count, cudaStream_t stream)
{
    const size_t smem = sizeof(int32_t) * ROUTE_WARPS * (size_t) n_experts;
    cudaError_t err = cudaFuncSetAttribute(route_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int) sizeof(int32_t) * ROUTE_WARPS * kMaxExperts);
    if (err != cudaSuccess) return set_cuda_error("route_sort: cudaFuncSetAttribute", err);
    route_sort_kernel<<<1, ROUTE_THREADS, smem, stream>>>(
        ids, ids_i64, weights, wdtype, T * topk, topk, n_experts, max_blocks, token_sorted,
        reinterpret_cast<__half*>(weight_sorted), expert_of_row, counts, expert_row0, block_expert, block_row0,
        meta, invalid_count);
    return check_launch("route_sort");
}

int launch_build_blocks(const int32_t* counts, int n_experts, int32_t* block_expert, int32_t* block_row0,
                        int max_blocks, int32_t* meta, cudaStream_t stream)
{
    build_blocks_kernel<<<1, ROUTE_THREADS, 0, stream>>>(counts, n_experts, max_blocks, block_expert, block_row0, meta);
    return check_launch("build_blocks");
}

}  // namespace exl3b
