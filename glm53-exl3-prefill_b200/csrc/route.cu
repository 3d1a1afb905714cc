// route.cu — expert sort and per-expert M-block table (stage 1 of the grouped prefill).
//
// route_hist_kernel + route_scatter_kernel replace the host-side torch sequence of
// kernel/exl3_grouped_runtime.py:59-67 (stable argsort by expert, token/weight/expert arrays, bincount,
// exclusive cumsum) AND the build_blocks launch of :72 with two launches over 2048-id chunks: chunk
// histograms into a small caller-provided scratch array, then one CTA per chunk ranks and scatters.
// Results are bit-identical to the reference: the sort is a stable counting sort (chunk order, then
// warp order inside a chunk, then lane order inside a 32-id batch).
//
// build_blocks_kernel keeps the reference's own entry point (kernel/exl3_grouped_prefill.cu:63-96,
// host fn :285-294) with the serial scan replaced by a block-wide parallel scan.
#include <cstdint>
#include <mutex>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "exl3_internal.h"

namespace exl3b {

namespace {

constexpr int ROUTE_THREADS = 1024;
constexpr int ROUTE_WARPS = ROUTE_THREADS / 32;
constexpr int ROUTE_BATCHES = 2;                               // 32-id batches per warp and chunk
constexpr int ROUTE_CHUNK = ROUTE_WARPS * 32 * ROUTE_BATCHES;  // flat ids per chunk (one CTA)
constexpr int HIST_THREADS = 256;

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

// Pass A: per-chunk expert histograms.  Chunk c covers flat ids [c*ROUTE_CHUNK, (c+1)*ROUTE_CHUNK);
// hist[c*(E+1) + e] = routes of chunk c to expert e, hist[c*(E+1) + E] = ids outside [0, E).
__global__ __launch_bounds__(HIST_THREADS)
void route_hist_kernel(const void* __restrict__ ids, int ids_i64, int64_t R, int n_experts, int32_t* __restrict__ hist)
{
    extern __shared__ int32_t s_h[];                    // [E + 1]
    const int t = threadIdx.x, E = n_experts;
    for (int i = t; i <= E; i += HIST_THREADS) s_h[i] = 0;
    __syncthreads();
    const int64_t lo = (int64_t) blockIdx.x * ROUTE_CHUNK;
    const int64_t hi = min(R, lo + ROUTE_CHUNK);
    for (int64_t i = lo + t; i < hi; i += HIST_THREADS)
    {
        const int64_t e = load_id(ids, ids_i64, i);
        atomicAdd(&s_h[(e >= 0 && e < E) ? (int) e : E], 1);
    }
    __syncthreads();
    for (int i = t; i <= E; i += HIST_THREADS) hist[(int64_t) blockIdx.x * (E + 1) + i] = s_h[i];
}

// Routes of chunk cc to bucket e (E = ids outside [0, E)): the sum of the chunk's `parts` histogram rows
// (the router kernel writes one row per 128 tokens, so a 2048-id chunk may span several), rows past
// hist_rows counting zero.
__device__ __forceinline__ int chunk_count(const int32_t* __restrict__ hist, int cc, int e, int E, int parts,
                                           int64_t hist_rows)
{
    int v = 0;
    for (int q = 0; q < parts; ++q)
    {
        const int64_t h = (int64_t) cc * parts + q;
        if (h < hist_rows) v += hist[h * (E + 1) + e];
    }
    return v;
}

// Pass B: one CTA per chunk.  Every CTA derives, from the chunk histograms, the per-expert totals, the
// expert offsets (exclusive scan) and its own chunk's base; CTA 0 also writes counts, expert_row0,
// the block table and the invalid count.  Inside the chunk each warp owns ROUTE_CHUNK/32 consecutive
// ids; per-warp histograms (via __match_any_sync groups) give each warp its base per expert, and the
// scatter ranks equal ids by lane order, so the result is exactly a stable sort by expert.
__global__ __launch_bounds__(ROUTE_THREADS, 1)
void route_scatter_kernel(const void* __restrict__ ids, int ids_i64, const void* __restrict__ weights, int wdtype,
                          int64_t R, int topk, int n_experts, int max_blocks, const int32_t* __restrict__ hist,
                          int hist_parts, int64_t hist_rows,
                          int64_t* __restrict__ token_sorted, __half* __restrict__ weight_sorted,
                          int32_t* __restrict__ expert_of_row, int32_t* __restrict__ counts,
                          int32_t* __restrict__ expert_row0, int32_t* __restrict__ block_expert,
                          int32_t* __restrict__ block_row0, int32_t* __restrict__ meta,
                          int32_t* __restrict__ invalid_count)
{
    extern __shared__ int32_t whist[];                  // [ROUTE_WARPS][E]: per-warp counts, then bases
    __shared__ int s_warp[32];
    __shared__ int s_tot[2];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int E = n_experts;
    const int c = blockIdx.x, C = gridDim.x;

    // ---- totals, chunk base, expert offsets
    int total = 0, base = 0;
    if (t < E)
        for (int cc = 0; cc < C; ++cc)
        {
            const int v = chunk_count(hist, cc, t, E, hist_parts, hist_rows);
            total += v;
            base += (cc < c) ? v : 0;
        }
    const int row0 = block_scan_excl(t < E ? total : 0, s_warp, &s_tot[0]);
    const int n_valid = s_tot[0];
    if (c == 0)
    {
        if (t < E)
        {
            counts[t] = total;
            expert_row0[t] = row0;
        }
        write_block_table(total, E, max_blocks, block_expert, block_row0, meta, s_warp, s_tot);
        if (t == 0 && invalid_count)
        {
            int inv = 0;
            for (int cc = 0; cc < C; ++cc) inv += chunk_count(hist, cc, E, E, hist_parts, hist_rows);
            *invalid_count = inv;
        }
    }
    // rows left over by ids outside [0, E): token 0, expert 0, weight 0 (keeps later stages in bounds);
    // spread over every CTA, since in an expert-parallel sort most of the slots belong to other ranks
    for (int64_t i = (int64_t) n_valid + (int64_t) c * ROUTE_THREADS + t; i < R; i += (int64_t) C * ROUTE_THREADS)
    {
        token_sorted[i] = 0;
        weight_sorted[i] = __float2half(0.0f);
        expert_of_row[i] = 0;
    }

    // ---- per-warp histograms of this chunk
    for (int i = t; i < ROUTE_WARPS * E; i += ROUTE_THREADS) whist[i] = 0;
    __syncthreads();
    const int64_t wlo = (int64_t) c * ROUTE_CHUNK + warp * (ROUTE_CHUNK / ROUTE_WARPS);
    int key[ROUTE_BATCHES];
    __half wv[ROUTE_BATCHES];
    #pragma unroll
    for (int b = 0; b < ROUTE_BATCHES; ++b)
    {
        const int64_t i = wlo + b * 32 + lane;
        key[b] = -2;                                   // -2: past the end, -1: id outside [0, E)
        wv[b] = __float2half(0.0f);
        if (i < R)
        {
            const int64_t e = load_id(ids, ids_i64, i);
            key[b] = (e >= 0 && e < E) ? (int) e : -1;
            wv[b] = load_weight_f16(weights, wdtype, i);
        }
    }
    int32_t* my = whist + warp * E;
    unsigned peers[ROUTE_BATCHES];
    #pragma unroll
    for (int b = 0; b < ROUTE_BATCHES; ++b)
    {
        peers[b] = __match_any_sync(0xffffffffu, key[b]);
        if (key[b] >= 0 && lane == __ffs(peers[b]) - 1) my[key[b]] += __popc(peers[b]);
        __syncwarp();
    }
    __syncthreads();
    if (t < E)
    {
        int run = row0 + base;
        for (int w = 0; w < ROUTE_WARPS; ++w)
        {
            const int v = whist[w * E + t];
            whist[w * E + t] = run;
            run += v;
        }
    }
    __syncthreads();

    // ---- stable scatter
    const unsigned lt_mask = (1u << lane) - 1u;
    #pragma unroll
    for (int b = 0; b < ROUTE_BATCHES; ++b)
    {
        int pos = 0;
        if (key[b] >= 0) pos = my[key[b]] + __popc(peers[b] & lt_mask);
        __syncwarp();
        if (key[b] >= 0 && lane == __ffs(peers[b]) - 1) my[key[b]] += __popc(peers[b]);
        __syncwarp();
        if (key[b] >= 0)
        {
            const int64_t i = wlo + b * 32 + lane;
            token_sorted[pos] = i / topk;
            weight_sorted[pos] = wv[b];
            expert_of_row[pos] = key[b];
        }
    }
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

// The scatter kernel's shared-memory limit, raised once per device (with that device current), so that
// later calls only launch kernels (nothing but stream work while a stream is being captured).
namespace {

std::atomic<bool> g_scatter_attr_set[kMaxDevices] = {};

int scatter_attr_once()
{
    return once_per_device(g_scatter_attr_set, "route_sort", [](int) {
        const cudaError_t err = cudaFuncSetAttribute(route_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int) sizeof(int32_t) * ROUTE_WARPS * kMaxExperts);
        if (err != cudaSuccess) return set_cuda_error("route_sort: cudaFuncSetAttribute", err);
        return 0;
    });
}

}  // namespace

int64_t route_sort_scratch_elems(int64_t R, int n_experts)
{
    const int64_t chunks = R > 0 ? (R + ROUTE_CHUNK - 1) / ROUTE_CHUNK : 1;
    return chunks * (n_experts + 1);
}

int launch_route_sort(const void* ids, int ids_i64, const void* weights, int wdtype, int64_t T, int topk,
                      int n_experts, int max_blocks, int64_t* token_sorted, void* weight_sorted,
                      int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0, int32_t* block_expert,
                      int32_t* block_row0, int32_t* meta, int32_t* invalid_count, int32_t* scratch,
                      cudaStream_t stream)
{
    const int64_t R = T * topk;
    const int64_t chunks = R > 0 ? (R + ROUTE_CHUNK - 1) / ROUTE_CHUNK : 1;
    if (chunks > 0x7fffffffLL) return set_error("route_sort: too many routed rows");
    const size_t smem = sizeof(int32_t) * ROUTE_WARPS * (size_t) n_experts;
    int rc0 = scatter_attr_once();
    if (rc0) return rc0;
    route_hist_kernel<<<(unsigned) chunks, HIST_THREADS, sizeof(int32_t) * (n_experts + 1), stream>>>(
        ids, ids_i64, R, n_experts, scratch);
    int rc = check_launch("route_sort (histograms)");
    if (rc) return rc;
    route_scatter_kernel<<<(unsigned) chunks, ROUTE_THREADS, smem, stream>>>(
        ids, ids_i64, weights, wdtype, R, topk, n_experts, max_blocks, scratch, 1, chunks, token_sorted,
        reinterpret_cast<__half*>(weight_sorted), expert_of_row, counts, expert_row0, block_expert, block_row0,
        meta, invalid_count);
    return check_launch("route_sort (scatter)");
}

int64_t route_front_scratch_elems(int64_t T, int topk, int n_experts)
{
    const int64_t fused = router_tiles(T) * (n_experts + 1);
    const int64_t plain = route_sort_scratch_elems(T * topk, n_experts);
    return fused > plain ? fused : plain;
}

int launch_route_front(const void* x, int64_t T, int K, const void* w_router, int n_experts, const float* bias,
                       int topk, int norm, float scale, int64_t* ids, float* weights, int max_blocks,
                       int64_t* token_sorted, void* weight_sorted, int32_t* expert_of_row, int32_t* counts,
                       int32_t* expert_row0, int32_t* block_expert, int32_t* block_row0, int32_t* meta,
                       int32_t* scratch, int32_t* status, cudaStream_t stream, int slot_rows)
{
    const int64_t R = T * topk;
    // slot_rows: token_sorted receives the routing slot t*topk + j of each sorted row instead of its token
    const int div = slot_rows ? 1 : topk;
    // the router writes one histogram row per 128 tokens (128 * topk ids); when that divides the sort's
    // chunk, the sort's own histogram pass is not needed
    const bool fused = (ROUTE_CHUNK % (128 * topk)) == 0;
    int rc = launch_router_topk(x, T, K, w_router, n_experts, bias, topk, norm, scale, ids, weights,
                                fused ? scratch : nullptr, status, stream);
    if (rc) return rc;
    if (!fused)
        return launch_route_sort(ids, 1, weights, 0, slot_rows ? R : T, div, n_experts, max_blocks, token_sorted,
                                 weight_sorted, expert_of_row, counts, expert_row0, block_expert, block_row0, meta,
                                 nullptr, scratch, stream);
    const int64_t chunks = R > 0 ? (R + ROUTE_CHUNK - 1) / ROUTE_CHUNK : 1;
    const size_t smem = sizeof(int32_t) * ROUTE_WARPS * (size_t) n_experts;
    rc = scatter_attr_once();
    if (rc) return rc;
    route_scatter_kernel<<<(unsigned) chunks, ROUTE_THREADS, smem, stream>>>(
        ids, 1, weights, 0, R, div, n_experts, max_blocks, scratch, ROUTE_CHUNK / (128 * topk), router_tiles(T),
        token_sorted, reinterpret_cast<__half*>(weight_sorted), expert_of_row, counts, expert_row0, block_expert,
        block_row0, meta, nullptr);
    return check_launch("route_front (scatter)");
}

int launch_build_blocks(const int32_t* counts, int n_experts, int32_t* block_expert, int32_t* block_row0,
                        int max_blocks, int32_t* meta, cudaStream_t stream)
{
    build_blocks_kernel<<<1, ROUTE_THREADS, 0, stream>>>(counts, n_experts, max_blocks, block_expert, block_row0, meta);
    return check_launch("build_blocks");
}

// ------------------------------------------------------------------------------------ allocation-free variant
// For callers that cannot allocate device memory on the prefill path: for example an engine that has
// already handed almost all of the GPU to its KV cache, or a host program that drives the plain C ABI
// and owns no device allocator.  The chunk histograms then live in this file-scope array instead of a
// caller buffer.  Every GPU that loads the library holds it (256 KiB) until the process exits; every
// call shares it, so calls that overlap on the GPU (other streams, other host threads) race on it.
// The histogram kernel rewrites every entry the scatter kernel reads, so nothing needs clearing
// between calls.
static __device__ __align__(256) int32_t g_route_static_scratch[kRouteStaticScratchElems];

namespace {
std::mutex g_static_scratch_mu;
int32_t* g_static_scratch_ptr[64] = {};
}  // namespace

int launch_route_sort_noalloc(const void* ids, int ids_i64, const void* weights, int wdtype, int64_t T, int topk,
                              int n_experts, int max_blocks, int64_t* token_sorted, void* weight_sorted,
                              int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0, int32_t* block_expert,
                              int32_t* block_row0, int32_t* meta, int32_t* invalid_count, cudaStream_t stream)
{
    const int64_t need = route_sort_scratch_elems(T * topk, n_experts);
    if (need > kRouteStaticScratchElems)
        return set_error("route_sort_noalloc: this routing needs %lld int32 of scratch, the built-in array holds %lld "
                         "(use exl3_route_sort with caller scratch)", (long long) need,
                         (long long) kRouteStaticScratchElems);
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return set_cuda_error("route_sort_noalloc: cudaGetDevice", err);
    if (dev < 0 || dev >= 64) return set_error("route_sort_noalloc: device ordinal %d out of range", dev);
    int32_t* scratch = nullptr;
    {
        // First call on a device (with that device current): the host-side symbol is only a stand-in,
        // so fetch the array's device address once and keep it.
        std::lock_guard<std::mutex> lock(g_static_scratch_mu);
        if (!g_static_scratch_ptr[dev])
        {
            void* p = nullptr;
            err = cudaGetSymbolAddress(&p, g_route_static_scratch);
            if (err != cudaSuccess) return set_cuda_error("route_sort_noalloc: cudaGetSymbolAddress", err);
            g_static_scratch_ptr[dev] = static_cast<int32_t*>(p);
        }
        scratch = g_static_scratch_ptr[dev];
    }
    return launch_route_sort(ids, ids_i64, weights, wdtype, T, topk, n_experts, max_blocks, token_sorted,
                             weight_sorted, expert_of_row, counts, expert_row0, block_expert, block_row0, meta,
                             invalid_count, scratch, stream);
}

}  // namespace exl3b
