// hadamard.cu — the two row-wise Hadamard stages of the grouped prefill (HBM-bound).
//
// row_had (kernel/exl3_grouped_prefill.cu:101-115, host fn :297-311):
//     dst[r, blk] = fp16( H128( src[token_sorted[r] or r, blk] (.) suh[expert_of_row[r], blk] ) / sqrt(128) )
// act_had (kernel/exl3_grouped_prefill.cu:118-141, host fn :313-322):
//     a = fp16( min(g, L) * sigmoid(min(g, L)) * clamp(u, -L, L) );  act[r, blk] = fp16( H128(a (.) suh_down[e]) / sqrt(128) )
//
// Expert parallelism (no reference counterpart).  Token t (global index) lives on rank t / tpr at row
// t % tpr; routing ids are expert positions, rank r owning [r*E/N, (r+1)*E/N).
//   ep_pull_rows     copies, once per rank, every other rank's token row that has a route to one of this
//                    rank's experts into a local [N*tpr, K] buffer (reads cross NVLink; a peer pointer per
//                    rank, mapped through CUDA IPC);
//   row_had (peer)   then gathers rows by routing slot s = t * topk + j from that buffer (or the rank's own
//                    token buffer) and records slot_row[s] = sorted row;
//   ep_combine_push  sums, per token, the weighted output rows of this rank's experts (y_local rows
//                    slot_row[t*topk + j], j ascending) and stores that one row, fp16 or fp32, into
//                    row (t % tpr) * N + rank of the owner's staging buffer: one NVLink row per
//                    (token, rank) pair instead of one per routing slot, 512 contiguous bytes per store
//                    instruction (the GEMM epilogue's thread-per-row stores would cross the link as
//                    16-byte pieces);
//   ep_combine_reduce sums, per token of this rank, the staging rows of the ranks holding any of its
//                    routed experts, in rank order (deterministic, fp32).
//
// Layout: one warp per row; each half-warp owns one 128-column block per step, each lane 8 consecutive
// columns (one 16-byte load/store).  The H128 is a radix-2 butterfly with stages h = 1, 2, 4 inside
// the thread and h = 8, 16, 32, 64 across lanes (__shfl_xor_sync), applied in that order so that the
// fp32 arithmetic matches the CPU oracle bit for bit.  Several column steps are loaded ahead to keep
// enough bytes in flight per SM.
#include <cstdint>
#include <cuda_fp16.h>

#include "common.cuh"
#include "exl3_internal.h"

namespace exl3b {

namespace {

constexpr int HAD_THREADS = 256;
constexpr int HAD_ROWS_PER_CTA = HAD_THREADS / 32;
constexpr int HAD_UNROLL = 4;          // 128-column blocks per half-warp loaded ahead

__device__ __forceinline__ void unpack8(const uint4& q, float (&v)[8])
{
    const __half2* h = reinterpret_cast<const __half2*>(&q);
    #pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8])
{
    uint4 q;
    __half2* h = reinterpret_cast<__half2*>(&q);
    #pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    return q;
}

// H128 over 16 lanes x 8 values (element index = (lane & 15) * 8 + i), unnormalised.
__device__ __forceinline__ void had128_halfwarp(float (&v)[8], int lane)
{
    #pragma unroll
    for (int h = 1; h < 8; h <<= 1)
    {
        #pragma unroll
        for (int i = 0; i < 8; ++i)
            if (!(i & h))
            {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
    }
    #pragma unroll
    for (int m = 1; m < 16; m <<= 1)
    {
        const bool upper = (lane & m) != 0;
        #pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = upper ? (p - v[i]) : (v[i] + p);
        }
    }
}

enum RowSource : int { kRowsDirect = 0, kRowsGather = 1, kRowsPeer = 2 };

template <int SRC>
__global__ __launch_bounds__(HAD_THREADS)
void row_had_kernel(const __half* __restrict__ src, const PeerRows peers, __half* __restrict__ dst, int64_t rows,
                    int K, const int64_t* __restrict__ token_sorted, const int32_t* __restrict__ expert_of_row,
                    int expert_base, const __half* __restrict__ suh, int64_t suh_stride, int32_t* __restrict__ slot_row,
                    const int32_t* __restrict__ rows_dev)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (rows_dev != nullptr) rows = min(rows, (int64_t) __ldg(rows_dev));       // count known on the device only
    for (int64_t r = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; r < rows; r += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        const __half* in;
        if (SRC == kRowsPeer)
        {
            const int64_t slot = __ldg(token_sorted + r);
            const int64_t t = slot / peers.index_div;                           // routing slot -> token
            const int64_t rk = t / peers.rows_per_rank;
            if (slot_row != nullptr && lane == 0) slot_row[slot] = (int32_t) r;
            in = static_cast<const __half*>(peer_ptr(peers, rk)) + (t - rk * peers.rows_per_rank) * K;
        }
        else
            in = src + (SRC == kRowsGather ? __ldg(token_sorted + r) : r) * K;
        const __half* sc = suh + (int64_t) (__ldg(expert_of_row + r) - expert_base) * suh_stride;
        __half* out = dst + r * K;
        const int nblk = K / 128;
        const int hw = lane >> 4, col_in_blk = (lane & 15) * 8;

        for (int b0 = 0; b0 < nblk; b0 += 2 * HAD_UNROLL)
        {
            uint4 xq[HAD_UNROLL], sq[HAD_UNROLL];
            #pragma unroll
            for (int u = 0; u < HAD_UNROLL; ++u)
            {
                const int blk = b0 + 2 * u + hw;
                if (blk < nblk)
                {
                    xq[u] = __ldg(reinterpret_cast<const uint4*>(in + blk * 128 + col_in_blk));
                    sq[u] = __ldg(reinterpret_cast<const uint4*>(sc + blk * 128 + col_in_blk));
                }
                else
                {
                    xq[u] = make_uint4(0, 0, 0, 0);
                    sq[u] = make_uint4(0, 0, 0, 0);
                }
            }
            #pragma unroll
            for (int u = 0; u < HAD_UNROLL; ++u)
            {
                if (b0 + 2 * u >= nblk) break;                   // warp-uniform: no block for either half
                const int blk = b0 + 2 * u + hw;
                float v[8], s[8];
                unpack8(xq[u], v);
                unpack8(sq[u], s);
                #pragma unroll
                for (int i = 0; i < 8; ++i) v[i] *= s[i];
                had128_halfwarp(v, lane);
                #pragma unroll
                for (int i = 0; i < 8; ++i) v[i] *= HAD_SCALE;
                if (blk < nblk) *reinterpret_cast<uint4*>(out + blk * 128 + col_in_blk) = pack8(v);
            }
        }
    }
}

__global__ __launch_bounds__(HAD_THREADS)
void act_had_kernel(const __half* __restrict__ gu, __half* __restrict__ act, int64_t rows, int I,
                    const int32_t* __restrict__ expert_of_row, int expert_base, const __half* __restrict__ suh,
                    int64_t suh_stride, float limit, const int32_t* __restrict__ rows_dev)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (rows_dev != nullptr) rows = min(rows, (int64_t) __ldg(rows_dev));
    for (int64_t r = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; r < rows; r += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        const __half* g = gu + r * 2 * (int64_t) I;
        const __half* up = g + I;
        const __half* sc = suh + (int64_t) (__ldg(expert_of_row + r) - expert_base) * suh_stride;
        __half* out = act + r * (int64_t) I;
        const int nblk = I / 128;
        const int hw = lane >> 4, col_in_blk = (lane & 15) * 8;

        for (int b0 = 0; b0 < nblk; b0 += 2 * HAD_UNROLL)
        {
            uint4 gq[HAD_UNROLL], uq[HAD_UNROLL], sq[HAD_UNROLL];
            #pragma unroll
            for (int u = 0; u < HAD_UNROLL; ++u)
            {
                const int blk = b0 + 2 * u + hw;
                if (blk < nblk)
                {
                    gq[u] = __ldg(reinterpret_cast<const uint4*>(g + blk * 128 + col_in_blk));
                    uq[u] = __ldg(reinterpret_cast<const uint4*>(up + blk * 128 + col_in_blk));
                    sq[u] = __ldg(reinterpret_cast<const uint4*>(sc + blk * 128 + col_in_blk));
                }
                else
                {
                    gq[u] = make_uint4(0, 0, 0, 0);
                    uq[u] = make_uint4(0, 0, 0, 0);
                    sq[u] = make_uint4(0, 0, 0, 0);
                }
            }
            #pragma unroll
            for (int u = 0; u < HAD_UNROLL; ++u)
            {
                if (b0 + 2 * u >= nblk) break;
                const int blk = b0 + 2 * u + hw;
                float gv[8], uv[8], s[8], v[8];
                unpack8(gq[u], gv);
                unpack8(uq[u], uv);
                unpack8(sq[u], s);
                #pragma unroll
                for (int i = 0; i < 8; ++i)
                {
                    // Same expression as the reference, with the same fast exp and divide it is compiled
                    // with (--use_fast_math, kernel/exl3_grouped_runtime.py:44).
                    const float gc = fminf(gv[i], limit);
                    const float uc = fminf(fmaxf(uv[i], -limit), limit);
                    const float a = __fdividef(gc, 1.0f + __expf(-gc)) * uc;
                    v[i] = __half2float(__float2half_rn(a)) * s[i];
                }
                had128_halfwarp(v, lane);
                #pragma unroll
                for (int i = 0; i < 8; ++i) v[i] *= HAD_SCALE;
                if (blk < nblk) *reinterpret_cast<uint4*>(out + blk * 128 + col_in_blk) = pack8(v);
            }
        }
    }
}

// Bit j set: routing slot t*topk + j goes to an expert position in [e0, e1) (this rank's experts).
// topk <= 32; the whole warp calls it.
__device__ __forceinline__ unsigned local_routes(const int64_t* __restrict__ ids, int64_t t, int topk, int lane,
                                                 int64_t e0, int64_t e1)
{
    bool mine = false;
    if (lane < topk)
    {
        const int64_t e = __ldg(ids + t * topk + lane);
        mine = e >= e0 && e < e1;
    }
    return __ballot_sync(0xffffffffu, mine);
}

// Rank owning expert position e (0 <= e < E): rank r owns [r*E/N, (r+1)*E/N).
__device__ __forceinline__ int owner_rank(int64_t e, int n_experts, int n_ranks)
{
    int r = 0;
    while (r + 1 < n_ranks && e >= (int64_t) (r + 1) * n_experts / n_ranks) ++r;
    return r;
}

constexpr int EP_BATCH = 4;            // column steps per lane loaded ahead (pull, push, reduce)

// x_pulled[t] = token row t of its owner rank, for every token of the other ranks with at least one
// route to this rank's experts: each needed row crosses NVLink once, however many of this rank's
// experts it is routed to.
__global__ __launch_bounds__(HAD_THREADS)
void ep_pull_rows_kernel(const PeerRows x, int n_ranks, int rank, int K, const int64_t* __restrict__ ids, int topk,
                         int64_t e0, int64_t e1, __half* __restrict__ x_pulled)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tpr = x.rows_per_rank, T_all = tpr * n_ranks;
    const int nvec = K / 8;                                  // 16-byte vectors per row
    for (int64_t t = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; t < T_all; t += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        const int64_t rk = t / tpr;
        if (rk == rank) continue;
        if (!local_routes(ids, t, topk, lane, e0, e1)) continue;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(peer_ptr(x, rk)) + (t - rk * tpr) * K);
        uint4* dst = reinterpret_cast<uint4*>(x_pulled + t * K);
        for (int c0 = lane; c0 < nvec; c0 += 32 * 2 * EP_BATCH)
        {
            uint4 v[2 * EP_BATCH];
            #pragma unroll
            for (int b = 0; b < 2 * EP_BATCH; ++b)
                if (c0 + 32 * b < nvec) v[b] = __ldg(src + c0 + 32 * b);
            #pragma unroll
            for (int b = 0; b < 2 * EP_BATCH; ++b)
                if (c0 + 32 * b < nvec) dst[c0 + 32 * b] = v[b];
        }
    }
}

// Load V consecutive floats (fp32 or fp16 storage) / store V fp32 or fp16 values.
template <bool F16, int V>
__device__ __forceinline__ void load_v(const void* base, int64_t idx, float (&v)[V])
{
    static_assert(V == (F16 ? 8 : 4), "fp16 rows move 8 columns per lane, fp32 rows 4");
    if constexpr (F16)
        unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(base) + idx)), v);
    else
    {
        const float4 q = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
}

// Combine, expert side: for every token t (of any rank) with routes to this rank's experts, the sum of
// its weighted output rows here (y_local rows slot_row[t*topk + j], j ascending, fp32) is stored once,
// as fp16 or fp32, into row (t % tpr) * n_ranks + rank of the staging buffer of t's owner.  One warp
// per token; each store instruction writes 512 contiguous bytes.
template <bool F16>
__global__ __launch_bounds__(HAD_THREADS)
void ep_combine_push_kernel(const float* __restrict__ y, int K, const int64_t* __restrict__ ids, int topk, int64_t e0,
                            int64_t e1, const int32_t* __restrict__ slot_row, const PeerRows staging, int n_ranks,
                            int rank)
{
    constexpr int V = F16 ? 8 : 4;
    constexpr int NB = EP_BATCH * 8 / V;                 // 16-byte stores per lane in flight
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tpr = staging.rows_per_rank, T_all = tpr * n_ranks;
    for (int64_t t = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; t < T_all; t += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        const unsigned m = local_routes(ids, t, topk, lane, e0, e1);
        if (!m) continue;
        const int my_row = (m >> lane & 1u) ? __ldg(slot_row + t * topk + lane) : 0;
        const int64_t rk = t / tpr;
        const int64_t dst_row = ((t - rk * tpr) * n_ranks + rank) * (int64_t) K;
        void* base = const_cast<void*>(peer_ptr(staging, rk));
        for (int c0 = lane * V; c0 < K; c0 += 32 * V * NB)
        {
            float acc[NB][V];
            #pragma unroll
            for (int b = 0; b < NB; ++b)
                #pragma unroll
                for (int i = 0; i < V; ++i) acc[b][i] = 0.0f;
            for (unsigned mm = m; mm; mm &= mm - 1u)
            {
                const int r = __shfl_sync(0xffffffffu, my_row, __ffs(mm) - 1);
                #pragma unroll
                for (int b = 0; b < NB; ++b)
                {
                    const int c = c0 + 32 * V * b;
                    if (c < K)
                    {
                        const float4* src = reinterpret_cast<const float4*>(y + (int64_t) r * K + c);
                        #pragma unroll
                        for (int q = 0; q < V / 4; ++q)
                        {
                            const float4 v = __ldg(src + q);
                            acc[b][4 * q] += v.x; acc[b][4 * q + 1] += v.y;
                            acc[b][4 * q + 2] += v.z; acc[b][4 * q + 3] += v.w;
                        }
                    }
                }
            }
            #pragma unroll
            for (int b = 0; b < NB; ++b)
            {
                const int c = c0 + 32 * V * b;
                if (c >= K) continue;
                if constexpr (F16)
                    *reinterpret_cast<uint4*>(static_cast<__half*>(base) + dst_row + c) = pack8(acc[b]);
                else
                    *reinterpret_cast<float4*>(static_cast<float*>(base) + dst_row + c) =
                        make_float4(acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
            }
        }
    }
    // the rows are complete and visible system-wide before the kernel ends, so the collective that
    // follows it hands them to their owners
    __threadfence_system();
}

// Combine, owner side: out[t] = sum over the ranks r holding any of t's routed experts (ascending r) of
// staging row t * n_ranks + r (fp32 accumulation).  Unrouted tokens get zeros.
template <bool F16>
__global__ __launch_bounds__(HAD_THREADS)
void ep_combine_reduce_kernel(const void* __restrict__ staging, const int64_t* __restrict__ ids, int64_t T, int topk,
                              int n_experts, int n_ranks, float* __restrict__ out, int K)
{
    constexpr int V = F16 ? 8 : 4;
    constexpr int NB = EP_BATCH * 8 / V;                 // 16-byte vectors per lane in flight (per rank)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t t = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; t < T; t += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        unsigned bit = 0;
        if (lane < topk)
        {
            const int64_t e = __ldg(ids + t * topk + lane);
            if (e >= 0 && e < n_experts) bit = 1u << owner_rank(e, n_experts, n_ranks);
        }
        const unsigned m = __reduce_or_sync(0xffffffffu, bit);
        for (int c0 = lane * V; c0 < K; c0 += 32 * V * NB)
        {
            float acc[NB][V];
            #pragma unroll
            for (int b = 0; b < NB; ++b)
                #pragma unroll
                for (int i = 0; i < V; ++i) acc[b][i] = 0.0f;
            for (unsigned mm = m; mm; mm &= mm - 1u)
            {
                const int64_t row = (t * n_ranks + (__ffs(mm) - 1)) * (int64_t) K;
                #pragma unroll
                for (int b = 0; b < NB; ++b)
                {
                    const int c = c0 + 32 * V * b;
                    if (c < K)
                    {
                        float v[V];
                        load_v<F16, V>(staging, row + c, v);
                        #pragma unroll
                        for (int i = 0; i < V; ++i) acc[b][i] += v[i];
                    }
                }
            }
            #pragma unroll
            for (int b = 0; b < NB; ++b)
            {
                const int c = c0 + 32 * V * b;
                if (c >= K) continue;
                #pragma unroll
                for (int q = 0; q < V / 4; ++q)
                    *reinterpret_cast<float4*>(out + t * K + c + 4 * q) =
                        make_float4(acc[b][4 * q], acc[b][4 * q + 1], acc[b][4 * q + 2], acc[b][4 * q + 3]);
            }
        }
    }
}

// Combine of the single-GPU down stage: the down GEMM has stored each routing slot's weighted row
// w * y at row t*topk + j of y (slot order); out[t] = (accumulate ? out[t] : 0) + the sum of token t's
// slot rows whose id is in [0, E), j ascending (fp32, deterministic).  One warp per token, each lane 4
// columns of NB 512-byte column steps in flight per slot row.
template <bool IDS64>
__global__ __launch_bounds__(HAD_THREADS)
void combine_slots_kernel(const float* __restrict__ y, const void* __restrict__ ids, int64_t T, int topk,
                          int n_experts, float* __restrict__ out, int K, int accumulate)
{
    constexpr int NB = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t t = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; t < T; t += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        bool valid = false;
        if (lane < topk)
        {
            const int64_t e = IDS64 ? __ldg(static_cast<const long long*>(ids) + t * topk + lane)
                                    : (int64_t) __ldg(static_cast<const int*>(ids) + t * topk + lane);
            valid = e >= 0 && e < n_experts;
        }
        const unsigned m = __ballot_sync(0xffffffffu, valid);
        for (int c0 = lane * 4; c0 < K; c0 += 32 * 4 * NB)
        {
            float4 acc[NB];
            #pragma unroll
            for (int b = 0; b < NB; ++b)
            {
                const int c = c0 + 32 * 4 * b;
                acc[b] = (accumulate && c < K) ? *reinterpret_cast<const float4*>(out + t * K + c)
                                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            for (unsigned mm = m; mm; mm &= mm - 1u)
            {
                const float* row = y + (t * topk + (__ffs(mm) - 1)) * (int64_t) K;
                float4 v[NB];
                #pragma unroll
                for (int b = 0; b < NB; ++b)
                {
                    const int c = c0 + 32 * 4 * b;
                    v[b] = c < K ? __ldg(reinterpret_cast<const float4*>(row + c)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
                #pragma unroll
                for (int b = 0; b < NB; ++b)
                {
                    acc[b].x += v[b].x; acc[b].y += v[b].y; acc[b].z += v[b].z; acc[b].w += v[b].w;
                }
            }
            #pragma unroll
            for (int b = 0; b < NB; ++b)
            {
                const int c = c0 + 32 * 4 * b;
                if (c < K) *reinterpret_cast<float4*>(out + t * K + c) = acc[b];
            }
        }
    }
}

// Persistent grid: enough CTAs to fill every SM a few times over, each warp striding over rows.
unsigned had_grid(int64_t rows)
{
    const int64_t need = (rows + HAD_ROWS_PER_CTA - 1) / HAD_ROWS_PER_CTA;
    const int64_t cap = (int64_t) device_sm_count() * 8;
    return (unsigned) (need < cap ? need : cap);
}

}  // namespace

int launch_row_had(const void* src, void* dst, int64_t rows, int K, const int64_t* token_sorted,
                   const int32_t* expert_of_row, const void* suh, int64_t suh_stride, int gather,
                   cudaStream_t stream)
{
    if (rows <= 0) return 0;
    const dim3 grid(had_grid(rows));
    const PeerRows none{};
    if (gather)
        row_had_kernel<kRowsGather><<<grid, HAD_THREADS, 0, stream>>>(
            (const __half*) src, none, (__half*) dst, rows, K, token_sorted, expert_of_row, 0, (const __half*) suh,
            suh_stride, nullptr, nullptr);
    else
        row_had_kernel<kRowsDirect><<<grid, HAD_THREADS, 0, stream>>>(
            (const __half*) src, none, (__half*) dst, rows, K, nullptr, expert_of_row, 0, (const __half*) suh, suh_stride,
            nullptr, nullptr);
    return check_launch("row_had");
}

int launch_ep_row_had(const PeerRows& peers, void* dst, int64_t rows, int K, const int64_t* token_sorted,
                      const int32_t* expert_of_row, int expert_base, const void* suh, int64_t suh_stride,
                      int32_t* slot_row, const int32_t* rows_dev, cudaStream_t stream)
{
    if (rows <= 0) return 0;
    const dim3 grid(had_grid(rows));
    row_had_kernel<kRowsPeer><<<grid, HAD_THREADS, 0, stream>>>(
        nullptr, peers, (__half*) dst, rows, K, token_sorted, expert_of_row, expert_base, (const __half*) suh, suh_stride,
        slot_row, rows_dev);
    return check_launch("ep_row_had");
}

int launch_ep_pull_rows(const PeerRows& x, int n_ranks, int rank, int K, const int64_t* ids, int topk, int64_t e0,
                        int64_t e1, void* x_pulled, cudaStream_t stream)
{
    const int64_t T_all = x.rows_per_rank * n_ranks;
    if (n_ranks <= 1 || T_all <= 0) return 0;
    // One CTA per SM keeps ~32 KB of loads in flight per SM, more than NVLink needs, and leaves room on
    // every SM for the routing sort that runs beside the pull on another stream: its scatter CTA (1024
    // threads x 48 registers) fits beside one pull CTA (256 x 48) in the 64 K registers, not beside two.
    unsigned grid = had_grid(T_all);
    const unsigned cap = (unsigned) device_sm_count();
    if (grid > cap) grid = cap;
    ep_pull_rows_kernel<<<grid, HAD_THREADS, 0, stream>>>(x, n_ranks, rank, K, ids, topk, e0, e1, (__half*) x_pulled);
    return check_launch("ep_pull_rows");
}

int launch_ep_combine_push(const float* y, int K, const int64_t* ids, int topk, int64_t e0, int64_t e1,
                           const int32_t* slot_row, const PeerRows& staging, int n_ranks, int rank, int f16,
                           cudaStream_t stream)
{
    const int64_t T_all = staging.rows_per_rank * n_ranks;
    if (T_all <= 0) return 0;
    const dim3 grid(had_grid(T_all));
    if (f16)
        ep_combine_push_kernel<true><<<grid, HAD_THREADS, 0, stream>>>(y, K, ids, topk, e0, e1, slot_row, staging,
                                                                       n_ranks, rank);
    else
        ep_combine_push_kernel<false><<<grid, HAD_THREADS, 0, stream>>>(y, K, ids, topk, e0, e1, slot_row, staging,
                                                                        n_ranks, rank);
    return check_launch("ep_combine_push");
}

int launch_ep_combine_reduce(const void* staging, int f16, const int64_t* ids, int64_t T, int topk, int n_experts,
                             int n_ranks, float* out, int K, cudaStream_t stream)
{
    if (T <= 0) return 0;
    const dim3 grid(had_grid(T));
    if (f16)
        ep_combine_reduce_kernel<true><<<grid, HAD_THREADS, 0, stream>>>(staging, ids, T, topk, n_experts, n_ranks,
                                                                         out, K);
    else
        ep_combine_reduce_kernel<false><<<grid, HAD_THREADS, 0, stream>>>(staging, ids, T, topk, n_experts, n_ranks,
                                                                          out, K);
    return check_launch("ep_combine_reduce");
}

int launch_combine_slots(const float* y, const void* ids, int ids_i64, int64_t T, int topk, int n_experts, float* out,
                         int K, int accumulate, cudaStream_t stream)
{
    if (T <= 0) return 0;
    const dim3 grid(had_grid(T));
    if (ids_i64)
        combine_slots_kernel<true><<<grid, HAD_THREADS, 0, stream>>>(y, ids, T, topk, n_experts, out, K, accumulate);
    else
        combine_slots_kernel<false><<<grid, HAD_THREADS, 0, stream>>>(y, ids, T, topk, n_experts, out, K, accumulate);
    return check_launch("combine_slots");
}

int launch_act_had(const void* gu, void* act, int64_t rows, int I, const int32_t* expert_of_row, int expert_base,
                   const void* suh, int64_t suh_stride, float limit, cudaStream_t stream, const int32_t* rows_dev)
{
    if (rows <= 0) return 0;
    const dim3 grid(had_grid(rows));
    act_had_kernel<<<grid, HAD_THREADS, 0, stream>>>((const __half*) gu, (__half*) act, rows, I, expert_of_row,
                                                     expert_base, (const __half*) suh, suh_stride, limit, rows_dev);
    return check_launch("act_had");
}

}  // namespace exl3b
