// trellis_thin.cu — the grouped trellis GEMM for M-tiles of at most 128 rows (thin experts), on sm_100a
// tensor cores with the decoded weights as the MMA's A operand in tensor memory.
//
// Same math and output modes as trellis_gemm.cu (kernel/exl3_grouped_prefill.cu:148-279): for every row r
// of a tile, y[r, cols] = H128(A[r, :] . W'_e[:, cols]) / sqrt(128) * svh_e[cols], then stored / scattered
// by the shared epilogue_row().  It takes the one-block M-tiles (an expert's last M-tile) of up to 96
// rows (thin_kernel_max_rows(): every expert of a decode-sized or 256-token chunk, about half the
// M-tiles of a Zipf-routed 8192-token chunk), where a decoded weight feeds few rows:
//
//   * the product is computed transposed, D^T[cols, rows] = W'^T[cols, K] . A^T[K, rows]: the 128 output
//     columns of a column group are the MMA's M, the tile's rows its N (16..128);
//   * the decoder warps write the decoded weights straight into TMEM (tcgen05.st, one weight column per
//     TMEM lane, K pairs packed per 32-bit column), the A operand of tcgen05.mma; the activation rows come
//     by TMA (32-row boxes, only as many as the tile has) into shared memory, the B operand.  The decoded
//     weights never go through shared memory: in the 256-row kernel they are written there and read back
//     by every MMA, which for a one-block tile is most of its shared-memory traffic.  The eight decoder
//     warps are two sets of four that take alternate stages, so that the two on one SM sub-partition are
//     a stage apart and their barrier waits overlap the other's decode;
//   * the packed weights stream into a 12-stage ring (96 KB in flight per SM): a thin tile reads fresh
//     weights from HBM every stage, and with the 3 stages of the 256-row kernel their latency, not the
//     decode, set the pace;
//   * the epilogue copies each column group's accumulator (rows x 128 fp32) from TMEM into shared memory,
//     releases TMEM to the next tile's MMAs after the last one, and runs the H128 butterfly of each row
//     in one thread from there (rows padded to 129 floats: conflict-free on both sides);
//   * tiles come from a device-wide counter through a shared-memory ring, as in trellis_gemm.cu.
//
// Every mbarrier wait is bounded (exl3_set_wait_limit_ns); on a timeout the kernel records the error,
// every role leaves its loop, the producers wait (bounded) for their copies, the MMA thread for its MMAs,
// TMEM is freed and the kernel returns.
#include <cstdint>
#include <cstdlib>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "exl3_internal.h"
#include "trellis_common.cuh"

namespace exl3b {

// Tile counters of this kernel's scheduler (pair = next tile, CTAs finished), as in trellis_gemm.cu.
constexpr int kThinSchedSlots = 64;
static __device__ unsigned g_thin_sched[2 * kThinSchedSlots];

namespace {

using namespace trellis;

constexpr int TS = 3;                              // stages: activation smem and TMEM A operand
// Packed-weight ring: a thin tile streams fresh weights from HBM every stage (no other M-tile of the
// expert reuses them from L2) and decodes a stage in ~900 cycles, so the copies must run many stages
// ahead of the decoders for their latency not to set the pace.
constexpr int PKS = 12;
// Decoder warps: two sets of four (one warp per TMEM lane quarter), taking alternate stages.
constexpr int T_DEC_WARPS = 8;
constexpr int T_DEC_PER_STAGE = 4;
constexpr int T_THREADS = 32 * (4 + T_DEC_WARPS + 4);   // WG0: producers, MMA, scheduler; decoders; epilogue WG
constexpr int T_EPI_WARP0 = 4 + T_DEC_WARPS;
constexpr int T_EPI_WARPS = 4;
constexpr int T_TRING = 4;
constexpr int T_TILE_READERS = 3 + T_DEC_WARPS + T_EPI_WARPS;
// setmaxnreg split; its total must fit the registers the CTA is launched with (checked on the host).
constexpr uint32_t T_REG_WG0 = 56;
constexpr uint32_t T_REG_DEC = 112;
constexpr uint32_t T_REG_EPI = 208;
constexpr uint32_t T_REG_TOTAL = 128 * T_REG_WG0 + 32 * T_DEC_WARPS * T_REG_DEC + 128 * T_REG_EPI;
static_assert(T_REG_TOTAL <= 65536, "register split exceeds the register file");
// setmaxnreg.dec may only lower and setmaxnreg.inc only raise a warp's count from the launch allocation.
constexpr uint32_t T_LAUNCH_REGS = (65536u / T_THREADS) & ~7u;
static_assert(T_REG_WG0 <= T_LAUNCH_REGS && T_REG_DEC <= T_LAUNCH_REGS && T_REG_EPI >= T_LAUNCH_REGS,
              "setmaxnreg direction: producer and decoder warps lower, the epilogue raises");
constexpr int T_BOX_ROWS = 32;                     // activation rows per TMA box
constexpr int T_MAX_ROWS = 128;
constexpr uint32_t T_BOX_BYTES = T_BOX_ROWS * BK * 2;            // 4 KB
constexpr uint32_t T_ACT_STAGE = T_MAX_ROWS * BK * 2;            // 16 KB
constexpr uint32_t T_PK_STAGE = 2 * BPK_CB_BYTES;                // 8 KB
constexpr int T_LD = 129;                          // floats per staged accumulator row
constexpr uint32_t T_OFF_PK = TS * T_ACT_STAGE;
constexpr uint32_t T_OFF_EPI = T_OFF_PK + PKS * T_PK_STAGE;
constexpr uint32_t T_SMEM = T_OFF_EPI + T_MAX_ROWS * T_LD * 4 + 1024;   // staging: one column group
constexpr uint32_t T_STATIC_SMEM_MAX = 2 * 4 * (kMaxExperts + 1) + 512;
static_assert(T_SMEM + T_STATIC_SMEM_MAX <= 232448, "shared memory budget");
// TMEM: A stage s, column group c at columns s*64 + c*32 (64 K = 32 columns of fp16 pairs);
// Accumulators from T_ACC_COL: a tile of <= 64 rows uses slot a (alternating per such tile), column group
// c at T_ACC_COL + a*128 + c*64, so that the next such tile's MMAs run while the epilogue drains it; a
// tile of 65..128 rows uses both slots, column group c at T_ACC_COL + c*128 (N <= 128 columns).
constexpr uint32_t T_TMEM_COLS = 512;
constexpr uint32_t T_ACC_COL = TS * 64;
constexpr int T_NARROW_ROWS = 64;
static_assert(T_ACC_COL + 256 <= T_TMEM_COLS, "TMEM A stages and accumulators exceed the allocation");

// Accumulator slots, kept identically by the MMA thread and the epilogue (same tiles, same order).
// Scalars only: an array indexed at run time would go to local memory.
struct ThinAcc {
    uint32_t use0 = 0, use1 = 0;    // tiles that have used slot 0 / slot 1
    uint32_t next = 0;              // slot of the next tile of <= 64 rows
    __device__ __forceinline__ uint32_t mask(bool wide) const { return wide ? 3u : 1u << next; }
    __device__ __forceinline__ uint32_t col(bool wide) const { return T_ACC_COL + (wide ? 0u : next * 128u); }
    __device__ __forceinline__ void advance(bool wide)
    {
        if (wide || next == 0) ++use0;
        if (wide || next == 1) ++use1;
        if (!wide) next ^= 1u;
    }
};

__device__ __forceinline__ bool thin_take_tile(uint32_t it, volatile int* s_tile, uint64_t* tile_full,
                                               uint64_t* tile_empty, volatile int* abort_flag, const GemmArgs& p,
                                               unsigned mask, bool arrive, int& t)
{
    const int slot = it % T_TRING;
    const bool ok = mbar_wait(&tile_full[slot], (it / T_TRING) & 1u, abort_flag, p.status, p.wait_ns);
    t = ok ? s_tile[slot] : -1;
    if (!__all_sync(mask, ok)) return false;
    if (arrive) mbar_arrive(&tile_empty[slot]);
    return t >= 0;
}

__global__ __launch_bounds__(T_THREADS, 1)
void trellis_thin_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ PackedMaps tmap_w,
                         const GemmArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t act_full[TS], dec_full[TS], mma_done[TS];
    __shared__ uint64_t pk_full[PKS], pk_empty[PKS];
    __shared__ uint64_t acc_full[2], acc_empty[2], bar_final;
    __shared__ uint64_t tile_full[T_TRING], tile_empty[T_TRING];
    __shared__ int s_tile_raw[T_TRING];
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_abort;
    __shared__ int s_two[kMaxExperts + 1], s_one[kMaxExperts + 1];
    __shared__ volatile int s_epi_go[T_EPI_WARPS];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int E = p.counts ? p.n_experts : 1;
    volatile int* s_tile = s_tile_raw;

    if (warp == 0)
    {
        mtile_prefix(p, E, s_two, s_one, lane);
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            for (int s = 0; s < TS; ++s)
            {
                mbar_init(&act_full[s], 1);
                mbar_init(&dec_full[s], T_DEC_PER_STAGE);
                mbar_init(&mma_done[s], 1);
            }
            for (int s = 0; s < PKS; ++s)
            {
                mbar_init(&pk_full[s], 1);
                mbar_init(&pk_empty[s], T_DEC_PER_STAGE);
            }
            for (int a = 0; a < 2; ++a)
            {
                mbar_init(&acc_full[a], 1);
                mbar_init(&acc_empty[a], T_EPI_WARPS);
            }
            mbar_init(&bar_final, 1);
            for (int s = 0; s < T_TRING; ++s)
            {
                mbar_init(&tile_full[s], 1);
                mbar_init(&tile_empty[s], T_TILE_READERS);
            }
            s_abort = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&s_tmem_base, T_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const uint32_t tmem_base = s_tmem_base;
    const int t_base = s_two[E] * p.n_tiles_n;     // the one-block tiles follow the two-block ones
    const int total_tiles = s_one[E] * p.n_tiles_n;
    volatile int* abort_flag = &s_abort;

    const int wg = warp >> 2;
    if (wg == 0)
    {
    setmaxnreg_dec<T_REG_WG0>();
    if (warp == 3)
    {
        // ================================================================ tile scheduler
        if (lane == 0)
        {
            unsigned* next_tile = &g_thin_sched[2 * p.sched_slot];
            for (uint32_t it = 0;; ++it)
            {
                const int slot = it % T_TRING;
                if (it >= T_TRING && !mbar_wait(&tile_empty[slot], ((it / T_TRING) & 1u) ^ 1u, abort_flag, p.status,
                                                p.wait_ns))
                    break;
                int t = (int) atomicAdd(next_tile, 1u);
                if (t >= total_tiles) t = -1;
                s_tile[slot] = t;
                mbar_arrive(&tile_full[slot]);
                if (t < 0) break;
            }
        }
    }
    else if (warp == 0)
    {
        // ================================================================ activation producer (B operand)
        if (lane == 0)
        {
            uint32_t g = 0;
            bool ok = true;
            int t;
            for (uint32_t it = 0; ok && thin_take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 1u, true, t); ++it)
            {
                const TileInfo ti = tile_info(p, s_two, s_one, E, t_base + t);
                const int nbox = (ti.rows + T_BOX_ROWS - 1) / T_BOX_ROWS;
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % TS;
                    if (g >= TS && !mbar_wait(&mma_done[s], ((g / TS) & 1u) ^ 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                    uint8_t* dst = smem + s * T_ACT_STAGE;
                    mbar_arrive_expect_tx(&act_full[s], nbox * T_BOX_BYTES);
                    for (int i = 0; i < nbox; ++i)
                        tma_load_2d(dst + i * T_BOX_BYTES, &tmap_a, kb * BK, ti.row_base + i * T_BOX_ROWS, &act_full[s]);
                }
            }
            for (uint32_t k = 0; k < TS && k < g; ++k)
            {
                const uint32_t gl = g - 1 - k;
                mbar_drain(&act_full[gl % TS], (gl / TS) & 1u, DRAIN_LIMIT_NS);
            }
        }
    }
    else if (warp == 2)
    {
        // ================================================================ packed-weight producer
        if (lane == 0)
        {
            uint32_t g = 0;
            bool ok = true;
            int t;
            for (uint32_t it = 0; ok && thin_take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 1u, true, t); ++it)
            {
                const TileInfo ti = tile_info(p, s_two, s_one, E, t_base + t);
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % PKS;
                    if (g >= PKS && !mbar_wait(&pk_empty[s], ((g / PKS) & 1u) ^ 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                    uint8_t* b_dst = smem + T_OFF_PK + s * T_PK_STAGE;
                    mbar_arrive_expect_tx(&pk_full[s], ti.ncb * BPK_CB_BYTES);
                    // one 4 KB tensor copy per column group: 8 trellis tiles x 4 k-tiles
                    for (int cb = 0; cb < ti.ncb; ++cb)
                        tma_load_4d(b_dst + cb * BPK_CB_BYTES, &tmap_w.m[ti.which[cb]], 0, ti.colblk[cb] * 8, kb * (BK / 16), ti.e,
                                    &pk_full[s]);
                }
            }
            for (uint32_t k = 0; k < PKS && k < g; ++k)
            {
                const uint32_t gl = g - 1 - k;
                mbar_drain(&pk_full[gl % PKS], (gl / PKS) & 1u, DRAIN_LIMIT_NS);
            }
        }
    }
    else
    {
        // ================================================================ MMA issuer (warp 1)
        // The issue of an M128 x K16 MMA returns only about as fast as the tensor pipe takes it (~80 cycles,
        // whatever N), so this thread keeps the work between MMAs short: the stage slot and phase are
        // counted, not divided out, both input barriers are tested in one round trip, and the bounded
        // waits run only when one of them is still pending.
        if (lane == 0)
        {
            uint32_t s = 0, ph = 0;                      // stage slot and its phase parity
            bool ok = true;
            int t;
            ThinAcc acc;
            const uint64_t b_desc0 = smem_desc_sw128(smem_u32(smem));
            for (uint32_t it = 0; ok && thin_take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 1u, true, t); ++it)
            {
                const TileInfo ti = tile_info(p, s_two, s_one, E, t_base + t);
                const int n_rows = (ti.rows + 15) & ~15;                  // MMA N: the tile's rows, 16..128
                const uint32_t idesc = idesc_f16_f32(128, n_rows);
                const bool wide = ti.rows > T_NARROW_ROWS;
                const uint32_t am = acc.mask(wide);
                // the epilogue has copied out the last accumulators held in this tile's slot(s)
                if ((am & 1u) && acc.use0 > 0 &&
                    !mbar_wait(&acc_empty[0], (acc.use0 - 1) & 1u, abort_flag, p.status, p.wait_ns)) break;
                if ((am & 2u) && acc.use1 > 0 &&
                    !mbar_wait(&acc_empty[1], (acc.use1 - 1) & 1u, abort_flag, p.status, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_col = tmem_base + acc.col(wide);
                const uint32_t d_cb = wide ? 128u : 64u;
                const int ncb = ti.ncb;
                for (int kb = 0; kb < p.num_kb; ++kb)
                {
                    if (!mbar_test_wait2(&act_full[s], &dec_full[s], ph) &&
                        (!mbar_wait(&act_full[s], ph, abort_flag, p.status, p.wait_ns) ||
                         !mbar_wait(&dec_full[s], ph, abort_flag, p.status, p.wait_ns))) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t b_desc = b_desc0 + (s * T_ACT_STAGE >> 4);   // descriptor address field: bytes / 16
                    const uint32_t a_col = tmem_base + s * 64;
                    #pragma unroll
                    for (int cb = 0; cb < 2; ++cb)
                    {
                        if (cb >= ncb) break;
                        #pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            umma_f16_tmem_a(d_col + cb * d_cb, a_col + cb * 32 + kk * 8, b_desc + 2 * kk, idesc,
                                            (kb | kk) != 0);
                    }
                    umma_commit(&mma_done[s]);               // activation slot and TMEM A stage free again
                    if (++s == TS) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                if (am & 1u) umma_commit(&acc_full[0]);
                if (am & 2u) umma_commit(&acc_full[1]);
                acc.advance(wide);
            }
            umma_commit(&bar_final);
            mbar_drain(&bar_final, 0, DRAIN_LIMIT_NS);
        }
    }
    }
    else if (warp < T_EPI_WARP0)
    {
        // ================================================================ decoders -> TMEM (A operand)
        // Two sets of four warps take alternate stages: warp w decodes the stages g with g % 2 = (w - 4) / 4,
        // both column groups.  The two warps of one SM sub-partition (w and w + 4) are then a stage apart,
        // so one decodes while the other is at its barriers; with both on the same stage (one column group
        // each) they reached their waits at the same moment and the sub-partition idled a third of the time.
        // Warp w owns TMEM lane quarter q = w % 4 (weight columns 32q .. 32q+31 of each column group).  Lane
        // l decodes column n = 32q + l: trellis tile column tn = n / 16, tile column n % 16, whose 16 K values
        // come from stream units 2(n%16) .. 2(n%16)+2.  Per column group and stage 4 tiles along K -> 64 K
        // values = 32 packed columns, written with one tcgen05.st.
        setmaxnreg_dec<T_REG_DEC>();
        const int q = warp & 3;
        const uint32_t par = static_cast<uint32_t>(warp - 4) >> 2;
        const int tn = 2 * q + (lane >> 4), nn = lane & 15;
        const DecodeConsts dk = p.dk;
        const uint32_t taddr_q = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        uint32_t g = 0;
        bool ok = true;
        int t;
        for (uint32_t it = 0; ok && thin_take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 0xffffffffu,
                                                   lane == 0, t); ++it)
        {
            const TileInfo ti = tile_info(p, s_two, s_one, E, t_base + t);
            for (int kb = 0; kb < p.num_kb; ++kb, ++g)
            {
                if ((g & 1u) != par) continue;
                const int s = g % TS, sp = g % PKS;
                // the packed rows have landed and the MMAs that read this TMEM stage before are done
                const bool ready = mbar_wait(&pk_full[sp], (g / PKS) & 1u, abort_flag, p.status, p.wait_ns) &&
                                   (g < TS || mbar_wait(&mma_done[s], ((g / TS) & 1u) ^ 1u, abort_flag, p.status,
                                                        p.wait_ns));
                if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                #pragma unroll
                for (int cb = 0; cb < 2; ++cb)
                {
                    if (cb >= ti.ncb) break;
                    const uint32_t* tile0 = reinterpret_cast<const uint32_t*>(smem + T_OFF_PK + sp * T_PK_STAGE +
                                                                             cb * BPK_CB_BYTES + tn * 128);
                    uint32_t u0[4], u1[4], u2[4];
                    #pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        const uint32_t* tile = tile0 + j * (BPK_ROW_BYTES / 4);
                        const uint2 ab = *reinterpret_cast<const uint2*>(tile + 2 * nn);
                        u0[j] = ab.x;
                        u1[j] = ab.y;
                        u2[j] = tile[(2 * nn + 2) & 31];
                    }
                    uint32_t r[32];
                    #pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        const uint4 lo = decode8(u0[j], u1[j], dk);   // K 16kt .. 16kt+7
                        const uint4 hi = decode8(u1[j], u2[j], dk);   // K 16kt+8 .. 16kt+15
                        r[8 * j + 0] = lo.x; r[8 * j + 1] = lo.y; r[8 * j + 2] = lo.z; r[8 * j + 3] = lo.w;
                        r[8 * j + 4] = hi.x; r[8 * j + 5] = hi.y; r[8 * j + 6] = hi.z; r[8 * j + 7] = hi.w;
                    }
                    tmem_st32(taddr_q + s * 64 + cb * 32, r);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                {
                    mbar_arrive(&pk_empty[sp]);
                    mbar_arrive(&dec_full[s]);
                }
            }
        }
    }
    else
    {
        // ================================================================ epilogue
        setmaxnreg_inc<T_REG_EPI>();
        const int q = warp & 3;
        const int et = threadIdx.x - T_EPI_WARP0 * 32;               // 0..127: the row this thread finishes
        float* S = reinterpret_cast<float*>(smem + T_OFF_EPI);
        ThinAcc acc;
        for (uint32_t it = 0;; ++it)
        {
            // The four warps meet at named barriers below, so they must leave the loop together: each
            // publishes whether it got the next tile and its accumulators, and all follow the joint answer.
            int t;
            bool got = thin_take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 0xffffffffu, lane == 0, t);
            // (t is -1 past the last tile: any in-range tile index keeps the lookups in bounds)
            const bool wide = tile_info(p, s_two, s_one, E, t_base + (t < 0 ? 0 : t)).rows > T_NARROW_ROWS;
            const uint32_t am = acc.mask(wide);
            if (got)
            {
                bool full = !(am & 1u) || mbar_wait(&acc_full[0], acc.use0 & 1u, abort_flag, p.status, p.wait_ns);
                full = full && (!(am & 2u) || mbar_wait(&acc_full[1], acc.use1 & 1u, abort_flag, p.status, p.wait_ns));
                got = __all_sync(0xffffffffu, full);
            }
            if (lane == 0) s_epi_go[q] = got ? 1 : 0;
            named_bar_sync(1, T_EPI_WARPS * 32);
            const bool go = s_epi_go[0] && s_epi_go[1] && s_epi_go[2] && s_epi_go[3];
            if (!go) break;
            const TileInfo ti = tile_info(p, s_two, s_one, E, t_base + t);
            tc_fence_after();
            // Per column group: TMEM -> shared memory (thread (q, lane) holds weight column 32q + lane for 32
            // rows per load), then each thread finishes one row.  The slot(s) go back to the MMAs once the last
            // column group is staged.
            const int nchunk = (ti.rows + 31) / 32;
            const uint32_t d_col = acc.col(wide);
            const uint32_t d_cb = wide ? 128u : 64u;
            for (int cb = 0; cb < ti.ncb; ++cb)
            {
                for (int c = 0; c < nchunk; ++c)
                {
                    uint32_t r[32];
                    tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + d_col + cb * d_cb + c * 32, r);
                    tmem_wait_ld();
                    float* col = S + (c * 32) * T_LD + q * 32 + lane;
                    #pragma unroll
                    for (int i = 0; i < 32; ++i)
                    {
                        asm volatile("" : "+r"(r[i]));
                        col[i * T_LD] = __uint_as_float(r[i]);
                    }
                }
                if (cb == ti.ncb - 1)
                {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)                                   // the slot's next tile may start
                    {
                        if (am & 1u) mbar_arrive(&acc_empty[0]);
                        if (am & 2u) mbar_arrive(&acc_empty[1]);
                    }
                }
                named_bar_sync(1, T_EPI_WARPS * 32);                 // every column of this group is staged
                if (et < ti.rows)
                {
                    float v[128];
                    const float* row = S + et * T_LD;
                    #pragma unroll
                    for (int c = 0; c < 128; ++c) v[c] = row[c];
                    epilogue_row(v, p, ti, cb, et);
                }
                named_bar_sync(1, T_EPI_WARPS * 32);                 // staging free for the next group
            }
            acc.advance(wide);
        }
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, T_TMEM_COLS);
    }
    else if (threadIdx.x == 0)
    {
        __threadfence();
        if (atomicAdd(&g_thin_sched[2 * p.sched_slot + 1], 1u) == gridDim.x - 1)
        {
            atomicExch(&g_thin_sched[2 * p.sched_slot], 0u);
            atomicExch(&g_thin_sched[2 * p.sched_slot + 1], 0u);
        }
    }
    // Launched behind the two-block kernel this grid may have started before that one ended: it does not
    // end before it, so that the next kernel on the stream sees both grids' results.
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

std::atomic<bool> g_thin_attr_set[kMaxDevices] = {};
std::atomic<unsigned> g_thin_launch_seq{0};

}  // namespace

// The largest one-block M-tile (an expert's last M-tile, 1..128 rows) this kernel takes; the larger
// ones run on the two-block kernel with one M-block.  0 = none (EXL3_B200_THIN_KERNEL=0); else
// EXL3_B200_THIN_MAX_ROWS, by default 96: at config 1 the tiles of 97..128 rows ran faster as one M-block
// of the two-block kernel (its MMAs cost N/2 cycles, the thin kernel's ~100 whatever N), at 64 and 96
// alike, below that the thin tiles' MMA issue saves more.  Read at every launch (two getenv per GEMM
// call), so a process can compare the kernels on one problem.
int thin_kernel_max_rows()
{
    const char* v = std::getenv("EXL3_B200_THIN_KERNEL");
    if (v && v[0] == '0') return 0;
    const char* m = std::getenv("EXL3_B200_THIN_MAX_ROWS");
    const int rows = m && m[0] ? std::atoi(m) : 96;
    return rows < 0 ? 0 : rows > 128 ? 128 : rows;
}

int launch_trellis_thin(const GemmArgs& args, const PackedMaps& maps, const void* a, int64_t a_rows, int grid,
                        bool after_two_block, cudaStream_t stream)
{
    CUtensorMap tmap;
    {
        const int rc = make_a_tensor_map(&tmap, a, a_rows, args.num_kb * BK, T_BOX_ROWS);
        if (rc) return rc;
    }
    GemmArgs p = args;
    p.sched_slot = (int) (g_thin_launch_seq.fetch_add(1, std::memory_order_relaxed) % kThinSchedSlots);
    const int rc = once_per_device(g_thin_attr_set, "trellis_thin", [](int) {
        cudaError_t err = cudaFuncSetAttribute(trellis_thin_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int) T_SMEM);
        if (err != cudaSuccess) return set_cuda_error("trellis_thin: cudaFuncSetAttribute", err);
        cudaFuncAttributes fa;
        err = cudaFuncGetAttributes(&fa, trellis_thin_kernel);
        if (err != cudaSuccess) return set_cuda_error("trellis_thin: cudaFuncGetAttributes", err);
        if ((uint32_t) fa.numRegs * T_THREADS < T_REG_TOTAL)
            return set_error("trellis_thin: kernel built with %d registers/thread, the split needs %u",
                             fa.numRegs, T_REG_TOTAL / T_THREADS);
        return 0;
    });
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(T_THREADS);
    cfg.dynamicSmemBytes = T_SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = after_two_block ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, trellis_thin_kernel, tmap, maps, p);
    if (err != cudaSuccess) return set_cuda_error("trellis_thin: launch", err);
    return check_launch("trellis_thin");
}

}  // namespace exl3b
