// trellis_common.cuh — device code shared by the 1-SM and 2-SM trellis GEMM kernels: the trellis
// decode, the tile table, the H128 epilogue and the output modes.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "exl3_internal.h"

namespace exl3b {
namespace trellis {

constexpr int BM = 128;                       // rows per M-block (UMMA M per CTA)
constexpr int BK = 64;                        // K per stage: one 128-byte swizzle atom of fp16
constexpr int CB = 128;                       // columns per H128 group
constexpr uint32_t A_BLOCK_BYTES = BM * BK * 2;                 // 16 KB
constexpr uint32_t BPK_ROW_BYTES = (CB / 16) * 128;             // 8 trellis tiles of one k-tile row: 1 KB
constexpr uint32_t BPK_CB_BYTES = (BK / 16) * BPK_ROW_BYTES;    // 4 KB per column group and stage
constexpr uint64_t DRAIN_LIMIT_NS = 50000000ull;                // 50 ms: copies / MMAs in flight at an abort

// QTIP 3INST computed code (Tseng et al. 2024): x = 89226354*s + 64248484, m = (x & 0x8fff8fff) ^ 0x3b603b60,
// weight = fp16 lo(m) + fp16 hi(m).  Decodes the 8 weights (one 16-byte K-run) of one lane.
// u0 = unit[lane], u1 = unit[(lane+1) % 32] of the tile's 1024-bit stream.
//
// The integer work is split between the logic pipe and the multiply-add pipe.  Each 32-bit window
// V = hi*2^16 + lo holds two states: x_hi = hi*A + B needs a shift, but x_lo = lo*A + B needs no mask,
// because t = V*A + B*(1 + 2^16) = x_lo + x_hi*2^16 (mod 2^32), so x_lo = t - x_hi*2^16 is two
// multiply-adds.  The mask-and-xor is one LOP3 per code word, and the fp16 sum of a word's halves is
// one half add; two sums are packed per 32-bit output word.
//
// The constants arrive as kernel parameters (DecodeConsts), not literals: with literals ptxas splits
// each mask-and-xor into two logic instructions (a LOP3 takes one immediate), which costs 8 extra
// logic-pipe instructions per 8 weights (44 instead of 52 instructions in all, and 26% more weights
// per cycle on sm_100a, measured).
struct DecodeConsts {
    uint32_t a, b, c, neg16, mask, flip;     // A, B, B*(1+2^16), 0xFFFF0000, 0x8fff8fff, 0x3b603b60
};

inline DecodeConsts decode_consts()
{
    constexpr uint32_t A = 89226354u, B = 64248484u;
    return DecodeConsts{A, B, B + (B << 16), 0xFFFF0000u, 0x8fff8fffu, 0x3b603b60u};
}

__device__ __forceinline__ uint4 decode8(uint32_t u0, uint32_t u1, const DecodeConsts& k)
{
    uint32_t v[4];
    v[0] = u0;
    asm("shf.l.wrap.b32 %0, %1, %2, 4;" : "=r"(v[1]) : "r"(u1), "r"(u0));
    asm("shf.l.wrap.b32 %0, %1, %2, 8;" : "=r"(v[2]) : "r"(u1), "r"(u0));
    asm("shf.l.wrap.b32 %0, %1, %2, 12;" : "=r"(v[3]) : "r"(u1), "r"(u0));
    uint32_t m[8];                                               // m[j]: masked code word of weight j
    #pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        uint32_t h, xh, t, xl;
        asm("shr.u32 %0, %1, 16;" : "=r"(h) : "r"(v[i]));
        asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(xh) : "r"(h), "r"(k.a), "r"(k.b));      // state bits [4i, 4i+16)
        asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(t) : "r"(v[i]), "r"(k.a), "r"(k.c));
        asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(xl) : "r"(xh), "r"(k.neg16), "r"(t));   // bits [4i+16, 4i+32)
        asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(m[i]) : "r"(xh), "r"(k.mask), "r"(k.flip));     // (a & b) ^ c
        asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(m[i + 4]) : "r"(xl), "r"(k.mask), "r"(k.flip));
    }
    uint32_t out[4];
    #pragma unroll
    for (int j = 0; j < 4; ++j)
        asm("{\n\t.reg .f16 al, ah, bl, bh, sa, sb;\n\t"
            "mov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
            "add.rn.f16 sa, al, ah;\n\tadd.rn.f16 sb, bl, bh;\n\t"
            "mov.b32 %0, {sa, sb};\n\t}" : "=r"(out[j]) : "r"(m[2 * j]), "r"(m[2 * j + 1]));
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// Decode one pipeline stage's share of one decoder warp.  The stage holds, per column group cb and
// k-tile kt, 8 trellis tiles (tile columns tn = 0..7) at Bpk offset (cb*4 + kt)*1024 + tn*128; warp wd
// owns tile column tn = wd of all of them (NQ = 4 per column group), so its NQ decodes are independent
// and are issued together.  The tile's stream position s (0..31) holds the 8 K-consecutive weights of
// N row n = s/2, K half s%2; they are written as one 16-byte chunk of the K-major SW128 layout:
// row n at (n/8)*1024 + (n%8)*128, chunk c = kt*2 + s%2 stored at slot c ^ (n%8).
//
// Lane l decodes stream position s(l) = 2*n(l) + l%2 with n(l) = 8*(l/16) + 2*((l/2)%4) + (l/8)%2, so
// the 8 lanes of each quarter-warp (one 128-byte shared-memory wavefront of a 16-byte store) cover
// the rows n%8 = {0,2,4,6} or {1,3,5,7} with both K halves: 8 distinct 16-byte slots, no bank conflict.
template <int NQ>
__device__ __forceinline__ void decode_stage(const uint8_t* bpk, uint8_t* bdec, int wd, int lane, const DecodeConsts& k)
{
    const int n = ((lane >> 4) << 3) | (((lane >> 1) & 3) << 1) | ((lane >> 3) & 1);
    const int s = 2 * n + (lane & 1);
    // the lane holding stream position s+1 (mod 32)
    const int s1 = (s + 1) & 31, n1 = s1 >> 1;
    const int src_lane = ((n1 >> 3) << 4) | ((n1 & 1) << 3) | (((n1 >> 1) & 3) << 1) | (s1 & 1);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(bpk + wd * 128) + s;
    uint32_t u0[NQ], u1[NQ];
    #pragma unroll
    for (int q = 0; q < NQ; ++q) u0[q] = src[q * 256];
    #pragma unroll
    for (int q = 0; q < NQ; ++q) u1[q] = __shfl_sync(0xffffffffu, u0[q], src_lane);
    const int r = n & 7;
    uint8_t* dst = bdec + (wd * 2 + (n >> 3)) * 1024 + r * 128;
    #pragma unroll
    for (int q = 0; q < NQ; ++q)
    {
        const uint4 w = decode8(u0[q], u1[q], k);
        const int chunk = (q & 3) * 2 + (lane & 1);
        *reinterpret_cast<uint4*>(dst + (q >> 2) * 16384 + ((chunk ^ r) << 4)) = w;
    }
}

struct GemmArgs {
    const uint16_t* packed[2];
    int64_t expert_stride_words;
    int tiles_n;
    const __half* svh[2];
    int64_t svh_stride;
    const int32_t* counts;
    const int32_t* expert_row0;
    int n_experts;
    int single_count;
    const int64_t* token_sorted;
    const __half* route_weight;
    void* out;
    int64_t out_ld;
    int mode;
    int gate_up;
    int n_cblocks;          // 128-column groups per source matrix
    int n_tiles_n;          // column tiles per M-tile
    int num_kb;             // K stages
    int64_t a_rows;         // rows of A (TMA boxes starting at or past this row are not issued)
    int32_t* status;
    DecodeConsts dk;        // trellis decode constants (see decode8)
    uint64_t wait_ns;       // limit of every bounded mbarrier wait (exl3_set_wait_limit_ns)
    int sched_slot;         // this launch's tile counter pair in the scheduler's device array
    int one_lo, one_hi;     // this launch's one-block M-tiles: an expert's last M-tile with rows in
                            // (one_lo, one_hi] (0..128: all of them; the rest go to the other kernel)
};

struct TileInfo {
    int e;
    int row_base;           // first sorted row of the tile
    int rows;               // valid rows (1..256)
    int nsub;               // M-blocks with rows (1 or 2)
    int ncb;                // column groups (1 or 2)
    int which[2];           // source matrix per column group
    int colblk[2];          // 128-column group index within the source matrix
    int out_col[2];         // first output column per column group
};

__device__ __forceinline__ int expert_count(const GemmArgs& p, int e)
{
    return p.counts ? __ldg(p.counts + e) : p.single_count;
}

__device__ __forceinline__ int expert_row0(const GemmArgs& p, int e)
{
    return p.expert_row0 ? __ldg(p.expert_row0 + e) : 0;
}

// Last e in [0, n) with prefix[e] <= v (prefix non-decreasing, prefix[0] = 0 <= v).
__device__ __forceinline__ int prefix_find(const int* prefix, int n, int v)
{
    int lo = 0, hi = n - 1;
    while (lo < hi)
    {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= v) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Column part of a tile: column tile nt of the source matrix (or matrices) -> column groups.
__device__ __forceinline__ void tile_columns(const GemmArgs& p, int nt, TileInfo& ti)
{
    const int N = p.n_cblocks * CB;
    if (p.gate_up)
    {
        ti.ncb = 2;
        ti.which[0] = 0; ti.colblk[0] = nt; ti.out_col[0] = nt * CB;
        ti.which[1] = 1; ti.colblk[1] = nt; ti.out_col[1] = N + nt * CB;
    }
    else
    {
        ti.ncb = min(2, p.n_cblocks - 2 * nt);
        ti.which[0] = 0; ti.colblk[0] = 2 * nt; ti.out_col[0] = 2 * nt * CB;
        ti.which[1] = 0; ti.colblk[1] = 2 * nt + 1; ti.out_col[1] = (2 * nt + 1) * CB;
    }
}

// Tile t of the longest-first schedule.  Every expert's rows are cut into M-tiles of up to 256 rows;
// an M-tile with more than 128 rows spans two 128-row M-blocks (two accumulators, twice the MMAs per
// decoded stage), one with at most 128 rows a single block.  The two-block M-tiles of all experts come
// first, in expert order, then the one-block M-tiles (only an expert's last M-tile can have <= 128
// rows; a launch takes those with a row count in (one_lo, one_hi]); column tiles run fastest, so the
// CTAs working at one time share an M-tile's A rows and an expert's packed weights in L2.  s_two /
// s_one: per-expert prefix counts of the two kinds of M-tile.
__device__ __forceinline__ TileInfo tile_info(const GemmArgs& p, const int* s_two, const int* s_one, int n_experts,
                                              int t)
{
    TileInfo ti;
    const int t2 = s_two[n_experts] * p.n_tiles_n;
    int mt, nt;
    if (t < t2)
    {
        mt = t / p.n_tiles_n;
        nt = t - mt * p.n_tiles_n;
        const int e = prefix_find(s_two, n_experts, mt);
        const int local = mt - s_two[e];
        ti.e = e;
        ti.row_base = expert_row0(p, e) + local * 256;
        ti.rows = min(256, expert_count(p, e) - local * 256);
        ti.nsub = 2;
    }
    else
    {
        const int u = t - t2;
        mt = u / p.n_tiles_n;
        nt = u - mt * p.n_tiles_n;
        const int e = prefix_find(s_one, n_experts, mt);
        const int cnt = expert_count(p, e);
        ti.e = e;
        ti.row_base = expert_row0(p, e) + (cnt / 256) * 256;
        ti.rows = cnt % 256;
        ti.nsub = 1;
    }
    tile_columns(p, nt, ti);
    return ti;
}

__device__ __forceinline__ void had128_inthread(float (&v)[128])
{
    #pragma unroll
    for (int h = 1; h < 128; h <<= 1)
    {
        #pragma unroll
        for (int i = 0; i < 128; ++i)
            if (!(i & h))
            {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
    }
}

// One accumulator row (128 columns) -> H128 * scale * svh -> store / scatter.
__device__ __forceinline__ void epilogue_row(float (&v)[128], const GemmArgs& p, const TileInfo& ti, int cb, int row)
{
    had128_inthread(v);
    const __half* svh = p.svh[ti.which[cb]] + (int64_t) ti.e * p.svh_stride + ti.colblk[cb] * CB;
    #pragma unroll
    for (int c = 0; c < 16; ++c)
    {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(svh) + c);
        const __half2* h = reinterpret_cast<const __half2*>(&q);
        #pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const float2 s = __half22float2(h[i]);
            float a = v[8 * c + 2 * i] * HAD_SCALE;
            float b = v[8 * c + 2 * i + 1] * HAD_SCALE;
            v[8 * c + 2 * i] = a * s.x;
            v[8 * c + 2 * i + 1] = b * s.y;
        }
    }
    const int64_t grow = (int64_t) ti.row_base + row;          // sorted row index
    const int col0 = ti.out_col[cb];
    if (p.mode == kModeStoreF16)
    {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.out) + grow * p.out_ld + col0);
        #pragma unroll
        for (int c = 0; c < 16; ++c)
        {
            uint4 q;
            __half2* h = reinterpret_cast<__half2*>(&q);
            #pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[8 * c + 2 * i], v[8 * c + 2 * i + 1]);
            dst[c] = q;
        }
    }
    else if (p.mode == kModeStoreF32)
    {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + grow * p.out_ld + col0);
        #pragma unroll
        for (int c = 0; c < 32; ++c) dst[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
    else
    {
        const float w = p.route_weight ? __half2float(p.route_weight[grow]) : 1.0f;
        if (p.mode == kModeStoreWeighted || p.mode == kModeStoreRows)
        {
            const int64_t drow = p.mode == kModeStoreRows ? __ldg(p.token_sorted + grow) : grow;
            float4* d4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + drow * p.out_ld + col0);
            #pragma unroll
            for (int c = 0; c < 32; ++c)
                d4[c] = make_float4(v[4 * c] * w, v[4 * c + 1] * w, v[4 * c + 2] * w, v[4 * c + 3] * w);
            return;
        }
        const int64_t tok = __ldg(p.token_sorted + grow);
        float* dst = reinterpret_cast<float*>(p.out) + tok * p.out_ld + col0;
        if (p.mode == kModeScatterAtomic)
        {
            #pragma unroll
            for (int c = 0; c < 32; ++c)
                red_add_v4(dst + 4 * c, v[4 * c] * w, v[4 * c + 1] * w, v[4 * c + 2] * w, v[4 * c + 3] * w);
        }
        else
        {
            float4* d4 = reinterpret_cast<float4*>(dst);
            #pragma unroll
            for (int c = 0; c < 32; ++c)
            {
                float4 o = d4[c];
                o.x += v[4 * c] * w; o.y += v[4 * c + 1] * w; o.z += v[4 * c + 2] * w; o.w += v[4 * c + 3] * w;
                d4[c] = o;
            }
        }
    }
}

// Per-expert counts of two-block M-tiles (rows in 129..256) and one-block M-tiles (rows in 1..128).
__device__ __forceinline__ void mtile_counts(int cnt, int one_lo, int one_hi, int& two, int& one)
{
    const int rem = cnt % 256;
    two = cnt / 256 + (rem > 128 ? 1 : 0);
    one = (rem > one_lo && rem <= one_hi) ? 1 : 0;
}

// Exclusive per-expert prefixes of both kinds of M-tile, computed by one warp into s_two[0..E] and
// s_one[0..E].
__device__ __forceinline__ void mtile_prefix(const GemmArgs& p, int E, int* s_two, int* s_one, int lane)
{
    const int per = (E + 31) / 32;
    const int base = lane * per;
    int sum2 = 0, sum1 = 0;
    for (int i = 0; i < per; ++i)
    {
        const int e = base + i;
        if (e < E)
        {
            int two, one;
            mtile_counts(expert_count(p, e), p.one_lo, p.one_hi, two, one);
            sum2 += two;
            sum1 += one;
        }
    }
    int inc2 = sum2, inc1 = sum1;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1)
    {
        const int y2 = __shfl_up_sync(0xffffffffu, inc2, o);
        const int y1 = __shfl_up_sync(0xffffffffu, inc1, o);
        if (lane >= o)
        {
            inc2 += y2;
            inc1 += y1;
        }
    }
    int run2 = inc2 - sum2, run1 = inc1 - sum1;
    for (int i = 0; i < per; ++i)
    {
        const int e = base + i;
        if (e < E)
        {
            s_two[e] = run2;
            s_one[e] = run1;
            int two, one;
            mtile_counts(expert_count(p, e), p.one_lo, p.one_hi, two, one);
            run2 += two;
            run1 += one;
        }
    }
    if (lane == 31)
    {
        s_two[E] = inc2;
        s_one[E] = inc1;
    }
}

// Host: the driver's tensor-map encoder, resolved once through the runtime.
inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn)
    {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// Host: 2-D fp16 tensor map over A [rows, K] with a 64 x box_rows box and the 128-byte swizzle.
inline int make_a_tensor_map(CUtensorMap* tmap, const void* a, int64_t rows, int K, int box_rows = BM)
{
    auto encode = get_encode_fn();
    if (!encode) return set_error("trellis_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t) K, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) K * 2};
    const cuuint32_t box[2] = {BK, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error("trellis_gemm: cuTensorMapEncodeTiled failed (%d)", (int) cr);
    return 0;
}

// The packed trellis words of both source matrices (gate, up; or the one matrix twice) as TMA tensor maps.
struct alignas(64) PackedMaps {
    CUtensorMap m[2];
};

// Host: 4-D tensor map over packed words [E][tiles_k][tiles_n][64] (int16, expert stride in words, which
// may exceed tiles_k*tiles_n*64 for the [E, 2, ...] gate / up views) with a 64 x 8 x 4 x 1 box: one
// column group's 8 trellis tiles of 4 k-tiles, a pipeline stage's 4 KB in one copy, landing in shared
// memory as [k-tile][tile][64 words] (1 KB per k-tile row).
inline int make_packed_tensor_map(CUtensorMap* tmap, const void* packed, int n_experts, int tiles_k, int tiles_n,
                                  int64_t expert_stride_words)
{
    auto encode = get_encode_fn();
    if (!encode) return set_error("trellis_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[4] = {64, (cuuint64_t) tiles_n, (cuuint64_t) tiles_k, (cuuint64_t) n_experts};
    const cuuint64_t strides[3] = {128, (cuuint64_t) tiles_n * 128, (cuuint64_t) expert_stride_words * 2};
    const cuuint32_t box[4] = {64, 8, (cuuint32_t) (BK / 16), 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult cr = encode(tmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(packed), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error("trellis_gemm: cuTensorMapEncodeTiled (packed weights) failed (%d)", (int) cr);
    return 0;
}

inline int make_packed_maps(PackedMaps* maps, const GemmArgs& p, int n_experts)
{
    for (int i = 0; i < 2; ++i)
    {
        const int rc = make_packed_tensor_map(&maps->m[i], p.packed[i], n_experts, p.num_kb * (BK / 16), p.tiles_n,
                                              p.expert_stride_words);
        if (rc) return rc;
    }
    return 0;
}

}  // namespace trellis

// The thin kernel (trellis_thin.cu): the one-block M-tiles of up to thin_kernel_max_rows() rows (96
// unless EXL3_B200_THIN_MAX_ROWS says otherwise); every other tile runs on trellis_gemm_kernel.
// EXL3_B200_THIN_KERNEL=0 sends every tile to trellis_gemm_kernel.
int thin_kernel_max_rows();
// after_two_block: launched right behind trellis_gemm_kernel on the same stream, so it may start on the
// SMs that kernel's CTAs leave (and ends only after that kernel has).
int launch_trellis_thin(const trellis::GemmArgs& args, const trellis::PackedMaps& maps, const void* a, int64_t a_rows,
                        int grid, bool after_two_block, cudaStream_t stream);

}  // namespace exl3b
