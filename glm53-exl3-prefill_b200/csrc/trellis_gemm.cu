// trellis_gemm.cu — weight-stationary grouped trellis GEMM on sm_100a tensor cores (tcgen05 + TMEM).
//
// Computes, for every routed expert e and every row r of e's sorted rows,
//     y[r, cols] = H128( A[r, :] . W'_e[:, cols] ) * (1/sqrt(128)) * svh_e[cols]       (fp32)
// and writes y as fp16 rows (gate|up stage), fp32 rows (fat GEMM), or scatters w[r] * y into
// out[token_sorted[r]] (down stage; atomic, or non-atomic for the single-expert fat GEMM).  This is
// the math of grouped_gemm_kernel<MODE> (kernel/exl3_grouped_prefill.cu:148-279) and of
// exl3_fat_gemm_v2_kernel (kernel/exl3_fat_gemm_v2.cu:72-234), re-designed for B200:
//
//   * persistent CTAs (one per SM) walk a static tile list; a tile is (expert, up to 256 rows,
//     up to 256 columns = two 128-column H128 groups);
//   * warp 0 streams A (activations, TMA 2-D tiled load into the 128-byte-swizzled K-major layout)
//     and the packed 4-bpw trellis tiles (bulk copies) into a 3-stage shared-memory ring;
//   * warps 2..9 decode each 16x16 trellis tile ONCE per tile into fp16 in the UMMA canonical
//     K-major SW128 layout; the decoded B stage feeds both 128-row M-blocks of the tile;
//   * warp 1 (one elected thread) issues tcgen05.mma kind::f16 (M=128, N=256, K=16) into TMEM
//     accumulators (2 x 256 fp32 columns) and commits each stage back to the ring;
//   * after the last K stage the same 8 warps drain TMEM (tcgen05.ld 32x32b: one thread owns one
//     row's 128 columns), release the accumulator to the MMA warp, and run the H128 butterfly,
//     the 1/sqrt(128) and svh scales and the store / scatter in registers.
//
// Every mbarrier wait is bounded in time (common.cuh); on a timeout the kernel records an error in
// the status word, every role leaves its loop, the MMA thread waits (bounded) for its MMAs, TMEM is
// freed and the kernel returns.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "exl3_internal.h"

namespace exl3b {

namespace {

constexpr int BM = 128;                       // rows per M-block (UMMA M)
constexpr int BK = 64;                        // K per stage: one 128-byte swizzle atom of fp16
constexpr int CB = 128;                       // columns per H128 group
constexpr int MAX_CB = 2;                     // column groups per tile (UMMA N <= 256)
constexpr int MB = 2;                         // M-blocks per tile sharing one decoded B stage
constexpr int STAGES = 3;
constexpr int NUM_DEC_WARPS = 8;
constexpr int THREADS = 64 + NUM_DEC_WARPS * 32;
constexpr uint32_t A_BLOCK_BYTES = BM * BK * 2;                 // 16 KB
constexpr uint32_t A_STAGE_BYTES = MB * A_BLOCK_BYTES;          // 32 KB
constexpr uint32_t BDEC_STAGE_BYTES = MAX_CB * CB * BK * 2;     // 32 KB
constexpr uint32_t BPK_ROW_BYTES = (CB / 16) * 128;             // 8 trellis tiles of one k-tile row: 1 KB
constexpr uint32_t BPK_CB_BYTES = (BK / 16) * BPK_ROW_BYTES;    // 4 KB
constexpr uint32_t BPK_STAGE_BYTES = MAX_CB * BPK_CB_BYTES;     // 8 KB
constexpr uint32_t OFF_BDEC = STAGES * A_STAGE_BYTES;
constexpr uint32_t OFF_BPK = OFF_BDEC + STAGES * BDEC_STAGE_BYTES;
constexpr uint32_t SMEM_BYTES = OFF_BPK + STAGES * BPK_STAGE_BYTES + 1024;   // + alignment slack
constexpr uint32_t TMEM_COLS = MB * 256;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;               // 2 s
constexpr uint64_t DRAIN_LIMIT_NS = 50000000ull;                // 50 ms (abort path)

static_assert(SMEM_BYTES <= 232448 - 4200, "shared memory budget");

// QTIP 3INST computed code (Tseng et al. 2024): x = 89226354*s + 64248484, m = (x & 0x8fff8fff) ^ 0x3b603b60,
// weight = fp16 lo(m) + fp16 hi(m).  Decodes the 8 weights (one 16-byte K-run) of one lane.
// u0 = unit[lane], u1 = unit[(lane+1) % 32] of the tile's 1024-bit stream.
__device__ __forceinline__ uint4 decode8(uint32_t u0, uint32_t u1)
{
    const uint32_t v0 = u0;
    const uint32_t v4 = __funnelshift_l(u1, u0, 4);
    const uint32_t v8 = __funnelshift_l(u1, u0, 8);
    const uint32_t v12 = __funnelshift_l(u1, u0, 12);
    uint32_t s[8] = {v0 >> 16, v4 >> 16, v8 >> 16, v12 >> 16, v0 & 0xffffu, v4 & 0xffffu, v8 & 0xffffu, v12 & 0xffffu};
    uint32_t m[8];
    #pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = ((s[j] * 89226354u + 64248484u) & 0x8fff8fffu) ^ 0x3b603b60u;
    uint32_t out[4];
    #pragma unroll
    for (int j = 0; j < 4; ++j)
    {
        const uint32_t lo = prmt(m[2 * j], m[2 * j + 1], 0x5410u);
        const uint32_t hi = prmt(m[2 * j], m[2 * j + 1], 0x7632u);
        __half2 h = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
        out[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// Decode one pipeline stage's share of one decoder warp.  The stage holds, per column group cb and
// k-tile kt, 8 trellis tiles (tile columns tn = 0..7) at Bpk offset (cb*4 + kt)*1024 + tn*128; warp wd
// owns tile column tn = wd of all of them (NQ = 4 per column group), so its NQ decodes are independent
// and are issued together.  Each lane writes its 8 K-consecutive weights of N row
// n = cb*128 + wd*16 + lane/2 as one 16-byte chunk of the K-major SW128 layout:
// row n at (n/8)*1024 + (n%8)*128, chunk c = kt*2 + lane%2 stored at slot c ^ (n%8).
template <int NQ>
__device__ __forceinline__ void decode_stage(const uint8_t* bpk, uint8_t* bdec, int wd, int lane)
{
    const uint32_t* src = reinterpret_cast<const uint32_t*>(bpk + wd * 128) + lane;
    uint32_t u0[NQ], u1[NQ];
    #pragma unroll
    for (int q = 0; q < NQ; ++q) u0[q] = src[q * 256];
    #pragma unroll
    for (int q = 0; q < NQ; ++q) u1[q] = __shfl_sync(0xffffffffu, u0[q], (lane + 1) & 31);
    const int r = (lane >> 1) & 7;
    uint8_t* dst = bdec + (wd * 2 + (lane >> 4)) * 1024 + r * 128;
    #pragma unroll
    for (int q = 0; q < NQ; ++q)
    {
        const uint4 w = decode8(u0[q], u1[q]);
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
    int32_t* status;
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

__device__ __forceinline__ TileInfo tile_info(const GemmArgs& p, const int* s_mt0, int n_experts, int t)
{
    TileInfo ti;
    const int mt = t / p.n_tiles_n;
    const int nt = t - mt * p.n_tiles_n;
    int lo = 0, hi = n_experts - 1;                  // last e with s_mt0[e] <= mt
    while (lo < hi)
    {
        const int mid = (lo + hi + 1) >> 1;
        if (s_mt0[mid] <= mt) lo = mid; else hi = mid - 1;
    }
    ti.e = lo;
    const int local = mt - s_mt0[lo];
    const int cnt = expert_count(p, lo);
    ti.row_base = expert_row0(p, lo) + local * (BM * MB);
    ti.rows = min(BM * MB, cnt - local * (BM * MB));
    ti.nsub = (ti.rows + BM - 1) / BM;
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
        const int64_t tok = __ldg(p.token_sorted + grow);
        const float w = p.route_weight ? __half2float(p.route_weight[grow]) : 1.0f;
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

__global__ __launch_bounds__(THREADS, 1)
void trellis_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const GemmArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_full[STAGES], bar_dec[STAGES], bar_empty[STAGES];
    __shared__ uint64_t bar_acc_full, bar_acc_empty, bar_final;
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_abort;
    __shared__ int s_mt0[kMaxExperts + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int E = p.counts ? p.n_experts : 1;

    // ---- per-expert M-tile prefix (warp 0), barriers (thread 32), TMEM (warp 1)
    if (warp == 0)
    {
        const int per = (E + 31) / 32;
        const int base = lane * per;
        int sum = 0;
        for (int i = 0; i < per; ++i)
        {
            const int e = base + i;
            if (e < E) sum += (expert_count(p, e) + BM * MB - 1) / (BM * MB);
        }
        int incl = sum;
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1)
        {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int run = incl - sum;
        for (int i = 0; i < per; ++i)
        {
            const int e = base + i;
            if (e < E)
            {
                s_mt0[e] = run;
                run += (expert_count(p, e) + BM * MB - 1) / (BM * MB);
            }
        }
        if (lane == 31) s_mt0[E] = incl;
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            for (int s = 0; s < STAGES; ++s)
            {
                mbar_init(&bar_full[s], 1);
                mbar_init(&bar_dec[s], NUM_DEC_WARPS);
                mbar_init(&bar_empty[s], 1);
            }
            mbar_init(&bar_acc_full, 1);
            mbar_init(&bar_acc_empty, NUM_DEC_WARPS);
            mbar_init(&bar_final, 1);
            s_abort = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&s_tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const uint32_t tmem_base = s_tmem_base;
    const int total_tiles = s_mt0[E] * p.n_tiles_n;
    volatile int* abort_flag = &s_abort;

    if (warp == 0)
    {
        // ================================================================ producer
        if (lane == 0)
        {
            uint32_t g = 0;
            for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x)
            {
                const TileInfo ti = tile_info(p, s_mt0, E, t);
                const uint16_t* src[2];
                for (int cb = 0; cb < ti.ncb; ++cb)
                    src[cb] = p.packed[ti.which[cb]] + (int64_t) ti.e * p.expert_stride_words + (int64_t) ti.colblk[cb] * 8 * 64;
                bool ok = true;
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1u;
                    if (g >= STAGES && !mbar_wait(&bar_empty[s], ph ^ 1u, abort_flag, p.status, WAIT_LIMIT_NS)) { ok = false; break; }
                    uint8_t* a_dst = smem + s * A_STAGE_BYTES;
                    uint8_t* b_dst = smem + OFF_BPK + s * BPK_STAGE_BYTES;
                    mbar_arrive_expect_tx(&bar_full[s], ti.nsub * A_BLOCK_BYTES + ti.ncb * BPK_CB_BYTES);
                    for (int sub = 0; sub < ti.nsub; ++sub)
                        tma_load_2d(a_dst + sub * A_BLOCK_BYTES, &tmap_a, kb * BK, ti.row_base + sub * BM, &bar_full[s]);
                    for (int cb = 0; cb < ti.ncb; ++cb)
                        for (int kt = 0; kt < BK / 16; ++kt)
                            bulk_load(b_dst + (cb * 4 + kt) * BPK_ROW_BYTES,
                                      src[cb] + (int64_t) (kb * 4 + kt) * p.tiles_n * 64, BPK_ROW_BYTES, &bar_full[s]);
                }
                if (!ok) break;
            }
            // Drain: every copy this thread issued must have landed before the CTA exits.
            for (uint32_t k = 0; k < STAGES && k < g; ++k)
            {
                const uint32_t gl = g - 1 - k;
                mbar_wait(&bar_full[gl % STAGES], (gl / STAGES) & 1u, abort_flag, p.status, DRAIN_LIMIT_NS);
            }
        }
    }
    else if (warp == 1)
    {
        // ================================================================ MMA issuer
        if (lane == 0)
        {
            uint32_t g = 0, tile_iter = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++tile_iter)
            {
                const TileInfo ti = tile_info(p, s_mt0, E, t);
                if (tile_iter > 0 && !mbar_wait(&bar_acc_empty, (tile_iter - 1) & 1u, abort_flag, p.status, WAIT_LIMIT_NS)) { ok = false; break; }
                tc_fence_after();
                const uint32_t idesc = idesc_f16_f32(BM, ti.ncb * CB);
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1u;
                    if (!mbar_wait(&bar_full[s], ph, abort_flag, p.status, WAIT_LIMIT_NS) ||
                        !mbar_wait(&bar_dec[s], ph, abort_flag, p.status, WAIT_LIMIT_NS)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * A_STAGE_BYTES);
                    const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + OFF_BDEC + s * BDEC_STAGE_BYTES));
                    for (int sub = 0; sub < ti.nsub; ++sub)
                    {
                        const uint64_t a_desc = smem_desc_sw128(a_addr + sub * A_BLOCK_BYTES);
                        #pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            umma_f16(tmem_base + sub * 256, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
                    }
                    umma_commit(&bar_empty[s]);
                }
                if (!ok) break;
                umma_commit(&bar_acc_full);
            }
            umma_commit(&bar_final);
            mbar_wait(&bar_final, 0, abort_flag, p.status, ok ? WAIT_LIMIT_NS : DRAIN_LIMIT_NS);
        }
    }
    else
    {
        // ================================================================ decoders + epilogue
        const int wd = warp - 2;
        const int quarter = warp & 3;                 // TMEM lanes this warp may access
        const int ecb = wd >> 2;                      // column group this warp drains
        uint32_t g = 0, tile_iter = 0;
        for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++tile_iter)
        {
            const TileInfo ti = tile_info(p, s_mt0, E, t);
            bool ok = true;
            for (int kb = 0; kb < p.num_kb; ++kb, ++g)
            {
                const int s = g % STAGES;
                const uint32_t ph = (g / STAGES) & 1u;
                if (!__all_sync(0xffffffffu, mbar_wait(&bar_full[s], ph, abort_flag, p.status, WAIT_LIMIT_NS))) { ok = false; break; }
                const uint8_t* bpk = smem + OFF_BPK + s * BPK_STAGE_BYTES;
                uint8_t* bdec = smem + OFF_BDEC + s * BDEC_STAGE_BYTES;
                if (ti.ncb == 2) decode_stage<8>(bpk, bdec, wd, lane);
                else decode_stage<4>(bpk, bdec, wd, lane);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_dec[s]);
            }
            if (!ok) break;
            if (!__all_sync(0xffffffffu, mbar_wait(&bar_acc_full, tile_iter & 1u, abort_flag, p.status, WAIT_LIMIT_NS))) break;
            tc_fence_after();
            for (int sub = 0; sub < ti.nsub; ++sub)
            {
                float v[128];
                if (ecb < ti.ncb)
                {
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + sub * 256 + ecb * CB;
                    uint32_t r0[32], r1[32], r2[32], r3[32];
                    tmem_ld32(taddr + 0, r0);
                    tmem_ld32(taddr + 32, r1);
                    tmem_ld32(taddr + 64, r2);
                    tmem_ld32(taddr + 96, r3);
                    tmem_wait_ld();
                    // The loaded registers are valid only after wait::ld; tie each one to a volatile
                    // statement after the wait so the compiler cannot hoist their uses above it.
                    #pragma unroll
                    for (int i = 0; i < 32; ++i)
                    {
                        asm volatile("" : "+r"(r0[i]), "+r"(r1[i]), "+r"(r2[i]), "+r"(r3[i]));
                        v[i] = __uint_as_float(r0[i]);
                        v[32 + i] = __uint_as_float(r1[i]);
                        v[64 + i] = __uint_as_float(r2[i]);
                        v[96 + i] = __uint_as_float(r3[i]);
                    }
                }
                if (sub == ti.nsub - 1)
                {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_acc_empty);
                }
                const int row = sub * BM + quarter * 32 + lane;
                if (ecb < ti.ncb && row < ti.rows) epilogue_row(v, p, ti, ecb, row);
            }
        }
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn()
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

bool g_attr_set[64] = {};

}  // namespace

int trellis_gemm_smem_bytes() { return (int) SMEM_BYTES; }

int launch_trellis_gemm(const GemmProblem& q, cudaStream_t stream)
{
    if (q.size_k % BK != 0 || q.size_k <= 0) return set_error("trellis_gemm: K must be a positive multiple of %d", BK);
    if (q.tiles_n % 8 != 0) return set_error("trellis_gemm: N must be a multiple of 128");
    if ((reinterpret_cast<uintptr_t>(q.a) & 15) != 0) return set_error("trellis_gemm: A must be 16-byte aligned");
    for (int i = 0; i < 2; ++i)
        if (q.packed[i] && (reinterpret_cast<uintptr_t>(q.packed[i]) & 15) != 0)
            return set_error("trellis_gemm: packed weights must be 16-byte aligned");
    if (q.expert_stride_words % 8 != 0) return set_error("trellis_gemm: expert stride must be a multiple of 8 words");
    if ((reinterpret_cast<uintptr_t>(q.out) & 15) != 0) return set_error("trellis_gemm: out must be 16-byte aligned");
    if (q.out_ld % 8 != 0) return set_error("trellis_gemm: output row stride must be a multiple of 8 elements");
    if (q.n_experts > kMaxExperts) return set_error("trellis_gemm: too many experts");
    if (q.a_rows <= 0) return 0;
    if (q.a_rows > 0x7fffffffLL) return set_error("trellis_gemm: too many rows");

    auto encode = get_encode_fn();
    if (!encode) return set_error("trellis_gemm: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tmap;
    const cuuint64_t dims[2] = {(cuuint64_t) q.size_k, (cuuint64_t) q.a_rows};
    const cuuint64_t strides[1] = {(cuuint64_t) q.size_k * 2};
    const cuuint32_t box[2] = {BK, BM};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(q.a), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error("trellis_gemm: cuTensorMapEncodeTiled failed (%d)", (int) cr);

    GemmArgs p;
    p.packed[0] = static_cast<const uint16_t*>(q.packed[0]);
    p.packed[1] = static_cast<const uint16_t*>(q.packed[1] ? q.packed[1] : q.packed[0]);
    p.expert_stride_words = q.expert_stride_words;
    p.tiles_n = q.tiles_n;
    p.svh[0] = static_cast<const __half*>(q.svh[0]);
    p.svh[1] = static_cast<const __half*>(q.svh[1] ? q.svh[1] : q.svh[0]);
    p.svh_stride = q.svh_stride;
    p.counts = q.counts;
    p.expert_row0 = q.expert_row0;
    p.n_experts = q.n_experts;
    p.single_count = q.single_count;
    p.token_sorted = q.token_sorted;
    p.route_weight = static_cast<const __half*>(q.route_weight);
    p.out = q.out;
    p.out_ld = q.out_ld;
    p.mode = q.mode;
    p.gate_up = q.gate_up;
    p.n_cblocks = q.tiles_n / 8;
    p.n_tiles_n = q.gate_up ? p.n_cblocks : (p.n_cblocks + 1) / 2;
    p.num_kb = q.size_k / BK;
    p.status = q.status;

    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return set_cuda_error("trellis_gemm: cudaGetDevice", err);
    if (dev < 64 && !g_attr_set[dev])
    {
        err = cudaFuncSetAttribute(trellis_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_BYTES);
        if (err != cudaSuccess) return set_cuda_error("trellis_gemm: cudaFuncSetAttribute", err);
        g_attr_set[dev] = true;
    }
    int grid = device_sm_count();
    if (!q.counts)
    {
        const int tiles = ((q.single_count + BM * MB - 1) / (BM * MB)) * p.n_tiles_n;
        if (tiles <= 0) return 0;
        grid = tiles < grid ? tiles : grid;
    }
    trellis_gemm_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(tmap, p);
    return check_launch("trellis_gemm");
}

}  // namespace exl3b
