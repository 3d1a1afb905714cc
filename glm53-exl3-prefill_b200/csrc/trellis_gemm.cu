// trellis_gemm.cu — weight-stationary grouped trellis GEMM on sm_100a tensor cores (tcgen05 + TMEM).
//
// Computes, for every routed expert e and every row r of e's sorted rows,
//     y[r, cols] = H128( A[r, :] . W'_e[:, cols] ) * (1/sqrt(128)) * svh_e[cols]       (fp32)
// and writes y as fp16 rows (gate|up stage), fp32 rows (fat GEMM), or scatters w[r] * y into
// out[token_sorted[r]] (down stage; atomic, or non-atomic for the single-expert fat GEMM).  This is
// the math of grouped_gemm_kernel<MODE> (kernel/exl3_grouped_prefill.cu:148-279) and of
// exl3_fat_gemm_v2_kernel (kernel/exl3_fat_gemm_v2.cu:72-234), re-designed for B200:
//
//   * persistent CTAs (one per SM, 512 threads) walk a static tile list; a tile is (expert, up to
//     256 rows, up to 256 columns = two 128-column H128 groups);
//   * warp 0 streams A (activations, TMA 2-D tiled load into the 128-byte-swizzled K-major layout)
//     into a 3-stage ring; warp 2 streams the packed 4-bpw trellis tiles (bulk copies) into their own
//     3-stage ring, refilled as soon as the decoders free a slot, so the HBM latency of the weights is
//     covered by up to six stages;
//   * warps 4..11 decode each 16x16 trellis tile ONCE per tile into fp16 in the UMMA canonical
//     K-major SW128 layout; the decoded B stage feeds both 128-row M-blocks of the tile;
//   * warp 1 (one elected thread) issues tcgen05.mma kind::f16 (M=128, N=256, K=16) into TMEM
//     accumulators (2 x 256 fp32 columns) and commits each stage back to the ring;
//   * warps 12..15 (the epilogue warpgroup, registers moved to it with setmaxnreg) drain TMEM after
//     the last K stage (tcgen05.ld 32x32b: one thread owns one row's 128 columns), release the
//     accumulator to the MMA thread, and run the H128 butterfly, the 1/sqrt(128) and svh scales
//     and the store / scatter in registers while the next tile's stages are loaded and decoded.
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
#include "trellis_common.cuh"

namespace exl3b {

namespace {

using namespace trellis;

constexpr int MAX_CB = 2;                     // column groups per tile (UMMA N <= 256)
constexpr int MB = 2;                         // M-blocks per tile sharing one decoded B stage
constexpr int STAGES = 3;
constexpr int NUM_DEC_WARPS = 8;
constexpr int NUM_EPI_WARPS = 4;
constexpr int THREADS = 512;                  // WG0: producer, MMA, 2 idle; WG1-2: decoders; WG3: epilogue
// setmaxnreg split: WG0 and the decoders give registers to the epilogue warpgroup.  setmaxnreg.inc
// waits until enough registers are free, so the split must fit the launch's 512 x 128 registers.
constexpr uint32_t REG_WG0 = 56, REG_DEC = 112, REG_EPI = 208;
constexpr uint32_t REG_TOTAL = 128 * REG_WG0 + 256 * REG_DEC + 128 * REG_EPI;
static_assert(REG_TOTAL <= 65536, "register split exceeds the register file");
constexpr uint32_t A_STAGE_BYTES = MB * A_BLOCK_BYTES;          // 32 KB
constexpr uint32_t BDEC_STAGE_BYTES = MAX_CB * CB * BK * 2;     // 32 KB
constexpr uint32_t BPK_STAGE_BYTES = MAX_CB * BPK_CB_BYTES;     // 8 KB
constexpr uint32_t OFF_BDEC = STAGES * A_STAGE_BYTES;
constexpr int PK_STAGES = 3;                  // packed-weight ring, refilled as soon as the decoders free a slot
constexpr uint32_t OFF_BPK = OFF_BDEC + STAGES * BDEC_STAGE_BYTES;
constexpr uint32_t SMEM_BYTES = OFF_BPK + PK_STAGES * BPK_STAGE_BYTES + 1024;   // + alignment slack
constexpr uint32_t TMEM_COLS = MB * 256;

static_assert(SMEM_BYTES <= 232448 - 4300, "shared memory budget");

__global__ __launch_bounds__(THREADS, 1)
void trellis_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const GemmArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_full[STAGES], bar_dec[STAGES], bar_empty[STAGES];
    __shared__ uint64_t pk_full[PK_STAGES], pk_empty[PK_STAGES];
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
        mtile_prefix(p, E, BM * MB, s_mt0, lane);
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
            for (int s = 0; s < PK_STAGES; ++s)
            {
                mbar_init(&pk_full[s], 1);
                mbar_init(&pk_empty[s], NUM_DEC_WARPS);
            }
            mbar_init(&bar_acc_full, 1);
            mbar_init(&bar_acc_empty, NUM_EPI_WARPS);
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

    const int wg = warp >> 2;
    if (wg == 0)
    {
    setmaxnreg_dec<REG_WG0>();
    if (warp == 0)
    {
        // ================================================================ A producer
        if (lane == 0)
        {
            uint32_t g = 0;
            for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x)
            {
                const TileInfo ti = tile_info(p, s_mt0, E, t, BM * MB, BM);
                bool ok = true;
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1u;
                    if (g >= STAGES && !mbar_wait(&bar_empty[s], ph ^ 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                    uint8_t* a_dst = smem + s * A_STAGE_BYTES;
                    mbar_arrive_expect_tx(&bar_full[s], ti.nsub * A_BLOCK_BYTES);
                    for (int sub = 0; sub < ti.nsub; ++sub)
                        tma_load_2d(a_dst + sub * A_BLOCK_BYTES, &tmap_a, kb * BK, ti.row_base + sub * BM, &bar_full[s]);
                }
                if (!ok) break;
            }
            // Drain: every copy this thread issued must have landed before the CTA exits.
            for (uint32_t k = 0; k < STAGES && k < g; ++k)
            {
                const uint32_t gl = g - 1 - k;
                mbar_drain(&bar_full[gl % STAGES], (gl / STAGES) & 1u, DRAIN_LIMIT_NS);
            }
        }
    }
    else if (warp == 2)
    {
        // ================================================================ packed-weight producer
        // The packed trellis rows come from HBM (each tile reads another expert column group), so they
        // have their own ring, refilled as soon as the decoders are done with a slot: the loads run up
        // to PK_STAGES stages ahead of the decoders, which run up to STAGES stages ahead of the MMAs.
        if (lane == 0)
        {
            uint32_t g = 0;
            for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x)
            {
                const TileInfo ti = tile_info(p, s_mt0, E, t, BM * MB, BM);
                const uint16_t* src[2];
                for (int cb = 0; cb < ti.ncb; ++cb)
                    src[cb] = p.packed[ti.which[cb]] + (int64_t) ti.e * p.expert_stride_words + (int64_t) ti.colblk[cb] * 8 * 64;
                bool ok = true;
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % PK_STAGES;
                    const uint32_t ph = (g / PK_STAGES) & 1u;
                    if (g >= PK_STAGES && !mbar_wait(&pk_empty[s], ph ^ 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                    uint8_t* b_dst = smem + OFF_BPK + s * BPK_STAGE_BYTES;
                    mbar_arrive_expect_tx(&pk_full[s], ti.ncb * BPK_CB_BYTES);
                    for (int cb = 0; cb < ti.ncb; ++cb)
                        for (int kt = 0; kt < BK / 16; ++kt)
                            bulk_load(b_dst + (cb * 4 + kt) * BPK_ROW_BYTES,
                                      src[cb] + (int64_t) (kb * 4 + kt) * p.tiles_n * 64, BPK_ROW_BYTES, &pk_full[s]);
                }
                if (!ok) break;
            }
            for (uint32_t k = 0; k < PK_STAGES && k < g; ++k)
            {
                const uint32_t gl = g - 1 - k;
                mbar_drain(&pk_full[gl % PK_STAGES], (gl / PK_STAGES) & 1u, DRAIN_LIMIT_NS);
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
                const TileInfo ti = tile_info(p, s_mt0, E, t, BM * MB, BM);
                if (tile_iter > 0 && !mbar_wait(&bar_acc_empty, (tile_iter - 1) & 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                tc_fence_after();
                const uint32_t idesc = idesc_f16_f32(BM, ti.ncb * CB);
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1u;
                    if (!mbar_wait(&bar_full[s], ph, abort_flag, p.status, p.wait_ns) ||
                        !mbar_wait(&bar_dec[s], ph, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
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
            // every MMA this thread issued has completed before TMEM is freed (on the abort path too)
            umma_commit(&bar_final);
            mbar_drain(&bar_final, 0, DRAIN_LIMIT_NS);
        }
    }
    }
    else if (wg < 3)
    {
        // ================================================================ decoders
        setmaxnreg_dec<REG_DEC>();
        const int wd = warp - 4;
        const DecodeConsts dk = p.dk;
        uint32_t g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x)
        {
            const TileInfo ti = tile_info(p, s_mt0, E, t, BM * MB, BM);
            for (int kb = 0; kb < p.num_kb; ++kb, ++g)
            {
                const int s = g % STAGES, sp = g % PK_STAGES;
                // the packed rows of this stage have landed, and the MMAs that read the decoded slot's
                // previous contents have completed
                const bool ready = mbar_wait(&pk_full[sp], (g / PK_STAGES) & 1u, abort_flag, p.status, p.wait_ns) &&
                                   (g < STAGES || mbar_wait(&bar_empty[s], ((g / STAGES) & 1u) ^ 1u, abort_flag, p.status,
                                                            p.wait_ns));
                if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                const uint8_t* bpk = smem + OFF_BPK + sp * BPK_STAGE_BYTES;
                uint8_t* bdec = smem + OFF_BDEC + s * BDEC_STAGE_BYTES;
                if (ti.ncb == 2) decode_stage<8>(bpk, bdec, wd, lane, dk);
                else decode_stage<4>(bpk, bdec, wd, lane, dk);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0)
                {
                    mbar_arrive(&pk_empty[sp]);
                    mbar_arrive(&bar_dec[s]);
                }
            }
        }
    }
    else
    {
        // ================================================================ epilogue
        // One warpgroup: warp w reads TMEM lanes 32*(w%4).. (its 32 accumulator rows) of every
        // (sub-block, column group), 128 columns per pass, releases the accumulator after the last
        // load, then finishes the pass in registers while the next tile's MMAs run.
        setmaxnreg_inc<REG_EPI>();
        const int quarter = warp & 3;
        uint32_t tile_iter = 0;
        for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++tile_iter)
        {
            const TileInfo ti = tile_info(p, s_mt0, E, t, BM * MB, BM);
            if (!__all_sync(0xffffffffu, mbar_wait(&bar_acc_full, tile_iter & 1u, abort_flag, p.status, p.wait_ns))) break;
            tc_fence_after();
            for (int sub = 0; sub < ti.nsub; ++sub)
            {
                for (int cb = 0; cb < ti.ncb; ++cb)
                {
                    float v[128];
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + sub * 256 + cb * CB;
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
                    if (sub == ti.nsub - 1 && cb == ti.ncb - 1)
                    {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bar_acc_empty);
                    }
                    const int row = sub * BM + quarter * 32 + lane;
                    if (row < ti.rows) epilogue_row(v, p, ti, cb, row);
                }
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

std::atomic<bool> g_attr_set[kMaxDevices] = {};

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

    CUtensorMap tmap;
    {
        const int rc = make_a_tensor_map(&tmap, q.a, q.a_rows, q.size_k);
        if (rc) return rc;
    }

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
    p.a_rows = q.a_rows;
    p.status = q.status;
    p.dk = decode_consts();
    p.wait_ns = wait_limit_ns();

    const int rc = once_per_device(g_attr_set, "trellis_gemm", [](int) {
        cudaError_t err = cudaFuncSetAttribute(trellis_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int) SMEM_BYTES);
        if (err != cudaSuccess) return set_cuda_error("trellis_gemm: cudaFuncSetAttribute", err);
        // setmaxnreg.inc in the epilogue warpgroup waits until the registers it asks for are free:
        // refuse to launch a build whose per-thread register count cannot cover the split.
        cudaFuncAttributes fa;
        err = cudaFuncGetAttributes(&fa, trellis_gemm_kernel);
        if (err != cudaSuccess) return set_cuda_error("trellis_gemm: cudaFuncGetAttributes", err);
        if ((uint32_t) fa.numRegs * THREADS < REG_TOTAL)
            return set_error("trellis_gemm: kernel built with %d registers/thread, the split needs %u",
                             fa.numRegs, REG_TOTAL / THREADS);
        return 0;
    });
    if (rc) return rc;
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
