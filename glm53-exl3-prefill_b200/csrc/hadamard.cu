// hadamard.cu — the two row-wise Hadamard stages of the grouped prefill (HBM-bound).
//
// row_had (kernel/exl3_grouped_prefill.cu:101-115, host fn :297-311):
//     dst[r, blk] = fp16( H128( src[token_sorted[r] or r, blk] (.) suh[expert_of_row[r], blk] ) / sqrt(128) )
// act_had (kernel/exl3_grouped_prefill.cu:118-141, host fn :313-322):
//     a = fp16( min(g, L) * sigmoid(min(g, L)) * clamp(u, -L, L) );  act[r, blk] = fp16( H128(a (.) suh_down[e]) / sqrt(128) )
//
// Expert parallelism (no reference counterpart): ep_row_had gathers each row straight from the memory of
// the GPU that owns the token (a peer pointer per rank, mapped through CUDA IPC): the sorted rows carry
// global routing slots s = t * topk + j, the token t = s / topk lives on rank t / tokens_per_rank at row
// t % tokens_per_rank, and the loads cross NVLink.  expert_base turns the global expert ids of the sorted
// rows into indices of this GPU's expert slice.  ep_push_rows copies each weighted output row of this
// rank's experts (stored locally by the down GEMM) into its routing slot of the token owner's staging
// buffer: one warp per row, 512 contiguous bytes per store instruction, so the NVLink writes are full
// packets (the GEMM epilogue's thread-per-row stores would cross the link as 16-byte pieces).
// ep_combine_reduce sums, for each of this rank's tokens, the topk rows in its staging buffer
// (slot t*topk + j), in slot order; slots whose routing id is outside [0, E) were never routed and are
// skipped.
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
                    int expert_base, const __half* __restrict__ suh, int64_t suh_stride)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t r = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; r < rows; r += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        const __half* in;
        if (SRC == kRowsPeer)
        {
            const int64_t t = __ldg(token_sorted + r) / peers.index_div;      // routing slot -> token
            const int64_t rk = t / peers.rows_per_rank;
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
                    int64_t suh_stride, float limit)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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

__global__ __launch_bounds__(HAD_THREADS)
void ep_combine_reduce_kernel(const float* __restrict__ staging, const int64_t* __restrict__ ids, int64_t T,
                              int topk, int n_experts, float* __restrict__ out, int N)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t t = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; t < T; t += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        uint32_t valid = 0;                              // bit j: slot j was routed
        for (int j = 0; j < topk; ++j)
        {
            const int64_t e = __ldg(ids + t * topk + j);
            if (e >= 0 && e < n_experts) valid |= 1u << j;
        }
        float4* dst = reinterpret_cast<float4*>(out + t * N);
        const float4* src = reinterpret_cast<const float4*>(staging + t * topk * (int64_t) N);
        for (int c = lane; c < N / 4; c += 32)
        {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j < topk; ++j)
                if (valid >> j & 1u)
                {
                    const float4 v = __ldg(src + (int64_t) j * (N / 4) + c);
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
            dst[c] = acc;
        }
    }
}

__global__ __launch_bounds__(HAD_THREADS)
void ep_push_rows_kernel(const float* __restrict__ y, int64_t rows, int N, const int64_t* __restrict__ slot_sorted,
                         const PeerRows staging)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t r = (int64_t) blockIdx.x * HAD_ROWS_PER_CTA + warp; r < rows; r += (int64_t) gridDim.x * HAD_ROWS_PER_CTA)
    {
        const int64_t slot = __ldg(slot_sorted + r) / staging.index_div;
        const int64_t rk = slot / staging.rows_per_rank;
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(const_cast<void*>(peer_ptr(staging, rk))) +
                                                (slot - rk * staging.rows_per_rank) * N);
        const float4* src = reinterpret_cast<const float4*>(y + r * N);
        #pragma unroll 4
        for (int c = lane; c < N / 4; c += 32) dst[c] = __ldg(src + c);
    }
    // the rows are complete and visible system-wide before the kernel ends, so the collective that
    // follows it hands them to their owners
    __threadfence_system();
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
            suh_stride);
    else
        row_had_kernel<kRowsDirect><<<grid, HAD_THREADS, 0, stream>>>(
            (const __half*) src, none, (__half*) dst, rows, K, nullptr, expert_of_row, 0, (const __half*) suh, suh_stride);
    return check_launch("row_had");
}

int launch_ep_row_had(const PeerRows& peers, void* dst, int64_t rows, int K, const int64_t* token_sorted,
                      const int32_t* expert_of_row, int expert_base, const void* suh, int64_t suh_stride,
                      cudaStream_t stream)
{
    if (rows <= 0) return 0;
    const dim3 grid(had_grid(rows));
    row_had_kernel<kRowsPeer><<<grid, HAD_THREADS, 0, stream>>>(
        nullptr, peers, (__half*) dst, rows, K, token_sorted, expert_of_row, expert_base, (const __half*) suh, suh_stride);
    return check_launch("ep_row_had");
}

int launch_ep_combine_reduce(const float* staging, const int64_t* ids, int64_t T, int topk, int n_experts,
                             float* out, int N, cudaStream_t stream)
{
    if (T <= 0) return 0;
    const dim3 grid(had_grid(T));
    ep_combine_reduce_kernel<<<grid, HAD_THREADS, 0, stream>>>(staging, ids, T, topk, n_experts, out, N);
    return check_launch("ep_combine_reduce");
}

int launch_ep_push_rows(const float* y, int64_t rows, int N, const int64_t* slot_sorted, const PeerRows& staging,
                        cudaStream_t stream)
{
    if (rows <= 0) return 0;
    const dim3 grid(had_grid(rows));
    ep_push_rows_kernel<<<grid, HAD_THREADS, 0, stream>>>(y, rows, N, slot_sorted, staging);
    return check_launch("ep_push_rows");
}

int launch_act_had(const void* gu, void* act, int64_t rows, int I, const int32_t* expert_of_row, int expert_base,
                   const void* suh, int64_t suh_stride, float limit, cudaStream_t stream)
{
    if (rows <= 0) return 0;
    const dim3 grid(had_grid(rows));
    act_had_kernel<<<grid, HAD_THREADS, 0, stream>>>((const __half*) gu, (__half*) act, rows, I, expert_of_row,
                                                     expert_base, (const __half*) suh, suh_stride, limit);
    return check_launch("act_had");
}

}  // namespace exl3b
