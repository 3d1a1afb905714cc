// trellis_gemm.cu — weight-stationary grouped trellis GEMM on sm_100a tensor cores (tcgen05 + TMEM).
//
// Computes, for every routed expert e and every row r of e's sorted rows,
//     y[r, cols] = H128( A[r, :] . W'_e[:, cols] ) * (1/sqrt(128)) * svh_e[cols]       (fp32)
// and writes y as fp16 rows (gate|up stage), fp32 rows (fat GEMM), stores w[r] * y at row r or at row
// token_sorted[r] (down stage), or scatters w[r] * y into out[token_sorted[r]] (atomic, or non-atomic
// for the single-expert fat GEMM).  This is the math of grouped_gemm_kernel<MODE>
// (kernel/exl3_grouped_prefill.cu:148-279) and of exl3_fat_gemm_v2_kernel (kernel/exl3_fat_gemm_v2.cu:
// 72-234), re-designed for B200:
//
//   * persistent CTAs (one per SM, 512 threads) take tiles from a device-wide counter in longest-first
//     order (tiles with two 128-row M-blocks, then tiles with one); one thread claims the next tile as
//     soon as a slot of a 4-entry shared-memory ring is free and every role reads the tiles from the
//     ring in the same order, so a CTA that finishes early takes more of the remaining work;
//   * a tile is (expert, up to 256 rows = two 128-row M-blocks, up to 256 columns = two 128-column H128
//     groups);
//   * warp 0 streams A (activations, TMA 2-D tiled load into the 128-byte-swizzled K-major layout)
//     into a 3-stage ring; warp 2 streams the packed 4-bpw trellis tiles (one 4-D TMA load of 4 KB per
//     column group and stage, straight from the [E, tiles_k, tiles_n, 64] layout) into their own 3-stage
//     ring, refilled as soon as the decoders free a slot;
//   * warps 4..11 decode each 16x16 trellis tile ONCE per tile into fp16 in the UMMA canonical
//     K-major SW128 layout; the decoded B stage feeds both 128-row M-blocks of the tile;
//   * warp 1 (one elected thread) issues tcgen05.mma kind::f16 (M=128, N=256, K=16) into TMEM.  TMEM
//     holds two 256-column accumulator slots: a two-block tile uses both, a one-block tile one of them
//     (alternating), so the epilogue of a one-block tile overlaps the next tile's MMAs, and each slot
//     goes back to the MMA thread as soon as the epilogue has read it;
//   * warps 12..15 (the epilogue warpgroup, registers moved to it with setmaxnreg) drain TMEM
//     (tcgen05.ld 32x32b: one thread owns one row's 128 columns) and run the H128 butterfly, the
//     1/sqrt(128) and svh scales and the store / scatter in registers.
//
// Every mbarrier wait is bounded in time (common.cuh; the limit is exl3_set_wait_limit_ns); on a
// timeout the kernel records an error in the status word, every role leaves its loop, the producers
// wait (bounded, ignoring the abort) for their copies in flight, the MMA thread for its MMAs, TMEM is
// freed and the kernel returns.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "exl3_internal.h"
#include "trellis_common.cuh"

namespace exl3b {

// Tile counters of the dynamic scheduler: pair i = (next tile, CTAs finished) of one launch.  A launch
// takes pair (launch sequence number % kSchedSlots), so launches that overlap on the GPU (other streams)
// use different counters unless kSchedSlots of them are in flight at once; the last CTA of a launch to
// finish puts both counters back to zero for the next launch that uses the pair.  Device code names the
// array directly; the host only passes the pair index.
constexpr int kSchedSlots = 64;
static __device__ unsigned g_gemm_sched[2 * kSchedSlots];

namespace {

using namespace trellis;

constexpr int MAX_CB = 2;                     // column groups per tile (UMMA N <= 256)
constexpr int MB = 2;                         // M-blocks per tile sharing one decoded B stage
constexpr int STAGES = 3;
constexpr int NUM_DEC_WARPS = 8;
constexpr int NUM_EPI_WARPS = 4;
constexpr int THREADS = 512;                  // WG0: A producer, MMA, packed producer, scheduler; WG1-2: decoders; WG3: epilogue
constexpr int TRING = 4;                      // tile ring entries
// Every role reads every tile from the ring: A producer, packed producer, MMA thread (one arrival each),
// the decoder warps and the epilogue warps (one arrival per warp).
constexpr int TILE_READERS = 3 + NUM_DEC_WARPS + NUM_EPI_WARPS;
// setmaxnreg split: WG0 and the decoders give registers to the epilogue warpgroup.  setmaxnreg.inc
// waits until enough registers are free, so the split must fit the launch's 512 x 128 registers.
constexpr uint32_t REG_WG0 = 56, REG_DEC = 112, REG_EPI = 208;
constexpr uint32_t REG_TOTAL = 128 * REG_WG0 + 256 * REG_DEC + 128 * REG_EPI;
static_assert(REG_TOTAL <= 65536, "register split exceeds the register file");
// setmaxnreg.dec may only lower and setmaxnreg.inc only raise a warp's count from the launch allocation.
static_assert(REG_WG0 <= 65536 / THREADS && REG_DEC <= 65536 / THREADS && REG_EPI >= 65536 / THREADS,
              "setmaxnreg direction: producer and decoder warps lower, the epilogue raises");
constexpr uint32_t A_STAGE_BYTES = MB * A_BLOCK_BYTES;          // 32 KB
constexpr uint32_t BDEC_STAGE_BYTES = MAX_CB * CB * BK * 2;     // 32 KB
constexpr uint32_t BPK_STAGE_BYTES = MAX_CB * BPK_CB_BYTES;     // 8 KB
constexpr uint32_t OFF_BDEC = STAGES * A_STAGE_BYTES;
constexpr int PK_STAGES = 3;                  // packed-weight ring, refilled as soon as the decoders free a slot
constexpr uint32_t OFF_BPK = OFF_BDEC + STAGES * BDEC_STAGE_BYTES;
constexpr uint32_t SMEM_BYTES = OFF_BPK + PK_STAGES * BPK_STAGE_BYTES + 1024;   // + alignment slack
constexpr uint32_t TMEM_COLS = 2 * 256;       // two accumulator slots of 256 fp32 columns
constexpr uint32_t STATIC_SMEM_MAX = 2 * 4 * (kMaxExperts + 1) + 512;   // M-tile prefixes + barriers, ring

static_assert(SMEM_BYTES + STATIC_SMEM_MAX <= 232448, "shared memory budget");

// Reads tile `it` of the ring (every role, in the same order): false on the end sentinel or an abort.
// Called by one thread (mask 1) or by all 32 lanes of a warp (mask ~0, result the same in every lane);
// `arrive` is set for exactly one thread per reader.
__device__ __forceinline__ bool take_tile(uint32_t it, volatile int* s_tile, uint64_t* tile_full,
                                          uint64_t* tile_empty, volatile int* abort_flag, const GemmArgs& p,
                                          unsigned mask, bool arrive, int& t)
{
    const int slot = it % TRING;
    const bool ok = mbar_wait(&tile_full[slot], (it / TRING) & 1u, abort_flag, p.status, p.wait_ns);
    t = ok ? s_tile[slot] : -1;
    if (!__all_sync(mask, ok)) return false;
    if (arrive) mbar_arrive(&tile_empty[slot]);
    return t >= 0;
}

// TMEM accumulator slots of the tiles in ring order.  A two-block tile uses slots 0 and 1 (M-block b in
// slot b); a one-block tile uses slot `nxt`, which alternates between one-block tiles and restarts at 0
// after a two-block tile (slot 0 is the one the epilogue releases first).  `uses` counts each slot's
// uses so far (the mbarrier phase).  The MMA thread and the epilogue keep one each and apply the same
// rule to the same tiles.  Scalars only: an array indexed at run time would go to local memory.
struct AccSlots {
    uint32_t uses0 = 0, uses1 = 0;
    int nxt = 0;
    int first = 0;                            // slot of the tile's first M-block

    __device__ __forceinline__ void start(const TileInfo& ti)
    {
        if (ti.nsub == 2)
        {
            first = 0;
            nxt = 0;
        }
        else
        {
            first = nxt;
            nxt ^= 1;
        }
    }
    __device__ __forceinline__ int slot(int sub) const { return sub == 0 ? first : 1; }
    __device__ __forceinline__ uint32_t uses(int a) const { return a == 0 ? uses0 : uses1; }
    __device__ __forceinline__ void used(int a)
    {
        if (a == 0) ++uses0; else ++uses1;
    }
};

__global__ __launch_bounds__(THREADS, 1)
void trellis_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ PackedMaps tmap_w,
                         const GemmArgs p)
{
    // The thin kernel launched behind this one reads none of its results, so its CTAs may take the SMs
    // that this grid's CTAs leave as they finish (programmatic dependent launch).
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_full[STAGES], bar_dec[STAGES], bar_empty[STAGES];
    __shared__ uint64_t pk_full[PK_STAGES], pk_empty[PK_STAGES];
    __shared__ uint64_t acc_full[2], acc_empty[2], bar_final;
    __shared__ uint64_t tile_full[TRING], tile_empty[TRING];
    __shared__ int s_tile_raw[TRING];
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_abort;
    __shared__ int s_two[kMaxExperts + 1], s_one[kMaxExperts + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int E = p.counts ? p.n_experts : 1;
    volatile int* s_tile = s_tile_raw;

    // ---- per-expert M-tile prefixes (warp 0), barriers (thread 32), TMEM (warp 1)
    if (warp == 0)
    {
        mtile_prefix(p, E, s_two, s_one, lane);
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
            for (int s = 0; s < 2; ++s)
            {
                mbar_init(&acc_full[s], 1);
                mbar_init(&acc_empty[s], NUM_EPI_WARPS);
            }
            for (int s = 0; s < TRING; ++s)
            {
                mbar_init(&tile_full[s], 1);
                mbar_init(&tile_empty[s], TILE_READERS);
            }
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
    const int total_tiles = (s_two[E] + s_one[E]) * p.n_tiles_n;
    volatile int* abort_flag = &s_abort;

    const int wg = warp >> 2;
    if (wg == 0)
    {
    setmaxnreg_dec<REG_WG0>();
    if (warp == 3)
    {
        // ================================================================ tile scheduler
        if (lane == 0)
        {
            unsigned* next_tile = &g_gemm_sched[2 * p.sched_slot];
            for (uint32_t it = 0;; ++it)
            {
                const int slot = it % TRING;
                if (it >= TRING && !mbar_wait(&tile_empty[slot], ((it / TRING) & 1u) ^ 1u, abort_flag, p.status,
                                              p.wait_ns))
                    break;
                int t = (int) atomicAdd(next_tile, 1u);
                if (t >= total_tiles) t = -1;
                s_tile[slot] = t;
                mbar_arrive(&tile_full[slot]);              // release: the tile index is visible to the readers
                if (t < 0) break;
            }
        }
    }
    else if (warp == 0)
    {
        // ================================================================ A producer
        if (lane == 0)
        {
            uint32_t g = 0;
            bool ok = true;
            int t;
            for (uint32_t it = 0; ok && take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 1u, true, t); ++it)
            {
                const TileInfo ti = tile_info(p, s_two, s_one, E, t);
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
            bool ok = true;
            int t;
            for (uint32_t it = 0; ok && take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 1u, true, t); ++it)
            {
                const TileInfo ti = tile_info(p, s_two, s_one, E, t);
                for (int kb = 0; kb < p.num_kb; ++kb, ++g)
                {
                    const int s = g % PK_STAGES;
                    const uint32_t ph = (g / PK_STAGES) & 1u;
                    if (g >= PK_STAGES && !mbar_wait(&pk_empty[s], ph ^ 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                    uint8_t* b_dst = smem + OFF_BPK + s * BPK_STAGE_BYTES;
                    mbar_arrive_expect_tx(&pk_full[s], ti.ncb * BPK_CB_BYTES);
                    // one 4 KB tensor copy per column group: 8 trellis tiles x 4 k-tiles
                    for (int cb = 0; cb < ti.ncb; ++cb)
                        tma_load_4d(b_dst + cb * BPK_CB_BYTES, &tmap_w.m[ti.which[cb]], 0, ti.colblk[cb] * 8, kb * (BK / 16), ti.e,
                                    &pk_full[s]);
                }
            }
            for (uint32_t k = 0; k < PK_STAGES && k < g; ++k)
            {
                const uint32_t gl = g - 1 - k;
                mbar_drain(&pk_full[gl % PK_STAGES], (gl / PK_STAGES) & 1u, DRAIN_LIMIT_NS);
            }
        }
    }
    else
    {
        // ================================================================ MMA issuer (warp 1)
        if (lane == 0)
        {
            uint32_t g = 0;
            AccSlots acc;
            bool ok = true;
            int t;
            for (uint32_t it = 0; ok && take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 1u, true, t); ++it)
            {
                const TileInfo ti = tile_info(p, s_two, s_one, E, t);
                acc.start(ti);
                const uint32_t idesc = idesc_f16_f32(BM, ti.ncb * CB);
                for (int kb = 0; kb < p.num_kb && ok; ++kb, ++g)
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
                        const int a = acc.slot(sub);
                        if (kb == 0 && acc.uses(a) > 0)
                        {
                            // the epilogue has read this slot's previous accumulator
                            if (!mbar_wait(&acc_empty[a], (acc.uses(a) - 1) & 1u, abort_flag, p.status, p.wait_ns)) { ok = false; break; }
                            tc_fence_after();
                        }
                        const uint64_t a_desc = smem_desc_sw128(a_addr + sub * A_BLOCK_BYTES);
                        #pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            umma_f16(tmem_base + a * 256, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
                    }
                    if (!ok) break;
                    umma_commit(&bar_empty[s]);
                }
                if (!ok) break;
                for (int sub = 0; sub < ti.nsub; ++sub)
                {
                    umma_commit(&acc_full[acc.slot(sub)]);
                    acc.used(acc.slot(sub));
                }
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
        int t;
        for (uint32_t it = 0; ok && take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 0xffffffffu, lane == 0, t); ++it)
        {
            const TileInfo ti = tile_info(p, s_two, s_one, E, t);
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
        // (M-block, column group), 128 columns per pass, releases an accumulator slot after its last
        // load, then finishes the pass in registers while the MMAs of the next tile run.
        setmaxnreg_inc<REG_EPI>();
        const int quarter = warp & 3;
        AccSlots acc;
        int t;
        bool ok = true;
        for (uint32_t it = 0; ok && take_tile(it, s_tile, tile_full, tile_empty, abort_flag, p, 0xffffffffu, lane == 0, t); ++it)
        {
            const TileInfo ti = tile_info(p, s_two, s_one, E, t);
            acc.start(ti);
            for (int sub = 0; sub < ti.nsub && ok; ++sub)
            {
                const int a = acc.slot(sub);
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[a], acc.uses(a) & 1u, abort_flag, p.status, p.wait_ns)))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int cb = 0; cb < ti.ncb; ++cb)
                {
                    float v[128];
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + a * 256 + cb * CB;
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
                    if (cb == ti.ncb - 1)
                    {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[a]);
                    }
                    const int row = sub * BM + quarter * 32 + lane;
                    if (row < ti.rows) epilogue_row(v, p, ti, cb, row);
                }
                acc.used(a);
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
    else if (threadIdx.x == 0)
    {
        // the last CTA of the launch to get here resets the scheduler's counters (every CTA has taken its
        // last tile by now)
        __threadfence();
        if (atomicAdd(&g_gemm_sched[2 * p.sched_slot + 1], 1u) == gridDim.x - 1)
        {
            atomicExch(&g_gemm_sched[2 * p.sched_slot], 0u);
            atomicExch(&g_gemm_sched[2 * p.sched_slot + 1], 0u);
        }
    }
}

std::atomic<bool> g_attr_set[kMaxDevices] = {};
std::atomic<unsigned> g_launch_seq{0};

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
    p.sched_slot = (int) (g_launch_seq.fetch_add(1, std::memory_order_relaxed) % kSchedSlots);

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
    // Two-block M-tiles (129..256 rows) on this kernel, and the one-block M-tiles (an expert's last M-tile,
    // 1..128 rows) with more than `thin_max` rows; those with 1..thin_max rows on the thin kernel, whose
    // decoded weights go straight to TMEM.  With counts on the device both kernels are launched (one of
    // them may find no tile of its kind); a single expert's row count decides on the host.
    const int thin_max = thin_kernel_max_rows();
    p.one_lo = thin_max;
    p.one_hi = BM;
    const int sms = device_sm_count();
    int grid_two = sms, grid_one = sms;
    bool run_two = true, run_one = thin_max > 0;
    // No expert has more rows than A: with at most thin_max rows in A every tile is the thin kernel's, and
    // launching the two-block kernel (TMEM set-up on every SM, no tile to take) would only delay it.  This
    // is every decode-sized call (one token: 8 rows).
    if (q.counts && run_one && q.a_rows <= thin_max) run_two = false;
    if (!q.counts)
    {
        const int rem = q.single_count % (BM * MB);
        const int n_two = q.single_count / (BM * MB) + (rem > BM ? 1 : 0) + (rem > thin_max && rem <= BM ? 1 : 0);
        const int n_one = (rem > 0 && rem <= thin_max) ? 1 : 0;
        const int t_two = n_two * p.n_tiles_n;
        const int t_one = n_one * p.n_tiles_n;
        run_two = t_two > 0;
        run_one = t_one > 0;
        grid_two = t_two < sms ? t_two : sms;
        grid_one = t_one < sms ? t_one : sms;
    }
    PackedMaps maps;
    {
        const int rc2 = make_packed_maps(&maps, p, q.counts ? q.n_experts : 1);
        if (rc2) return rc2;
    }
    if (run_two)
    {
        trellis_gemm_kernel<<<grid_two, THREADS, SMEM_BYTES, stream>>>(tmap, maps, p);
        const int rc2 = check_launch("trellis_gemm");
        if (rc2) return rc2;
    }
    if (run_one)
    {
        GemmArgs pt = p;
        pt.one_lo = 0;
        pt.one_hi = thin_max;
        return launch_trellis_thin(pt, maps, q.a, q.a_rows, grid_one, run_two, stream);
    }
    return 0;
}

}  // namespace exl3b
