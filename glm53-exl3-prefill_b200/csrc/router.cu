// router.cu — the routing front-end of a GLM-5.3-Flash MoE layer, fused into one sm_100a kernel.
//
// The reference takes topk_ids / topk_weights from vLLM's router and sorts them on the host
// (kernel/exl3_grouped_runtime.py:59-67, 86-112).  The router itself is the DeepSeek-V3 "noaux_tc"
// sigmoid router that GLM-5.3-Flash uses (docs/research/02-glm-5.3-flash-architecture.md:33:
// scoring_func sigmoid, topk_method noaux_tc, n_group = topk_group = 1, norm_topk_prob, routed_scaling_factor,
// fp32 router):
//     logits = x . Wr^T                      (fp32)
//     s      = sigmoid(logits)
//     ids    = the topk experts by s + e_score_correction_bias   (one group: the group step is a no-op)
//     w      = s[ids] / (sum s[ids] + 1e-20) * routed_scaling_factor   (the division only if norm)
//
// router_topk_kernel: one CTA per 128 tokens.
//   warp 0      TMA producer: per 64-wide K step, the x tile [128 x 64] and the router weight [E x 64]
//               (as nchunk boxes of `chunk` rows), 128-byte swizzle, into a ring of `stages` slots;
//   warp 1      TMEM owner and MMA issuer: D[128 x E] (fp32, E <= 512 TMEM columns) += x . Wr^T with
//               tcgen05.mma kind::f16 (fp16 x fp16 products are exact in fp32; only the accumulation
//               order differs from a CPU dot product);
//   warps 2..11 epilogue.  Warps 2..5 (thread = token = TMEM lane) turn the logits into sigmoid scores in
//               shared memory (the drained TMA ring); then all ten warps route the 128 tokens, one warp
//               per token: the lanes hold the selection scores s + bias of experts lane, lane + 32, ...,
//               and k rounds of a butterfly arg-max in the order (selection score descending, expert id
//               ascending) pick the experts; weights, ids and the tile's expert histogram (the route
//               sort's first pass, in shared memory) follow.  (A per-thread insertion top-k over all E
//               columns on four warps ran 6x slower: nearly every column made some lane of the warp
//               take the insertion path, and four warps could not hide the latency.)
// Every wait is bounded: on a timeout the kernel raises the CTA's abort flag, records the error in the
// status word, waits (bounded) for its own copies and MMAs in flight, frees TMEM and returns.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "exl3_internal.h"
#include "trellis_common.cuh"

namespace exl3b {

namespace {

constexpr int RT_BM = 128;                 // tokens per CTA (UMMA M, TMEM lanes)
constexpr int RT_BK = 64;                  // K per stage: one 128-byte swizzle atom of fp16
constexpr int RT_EPI_WARPS = 10;         // warps 2..11: scores (warps 2..5, one TMEM quarter each), routing
constexpr int RT_EPI_THREADS = RT_EPI_WARPS * 32;
constexpr int RT_THREADS = 64 + RT_EPI_THREADS;
constexpr int RT_MAX_STAGES = 6;
constexpr uint32_t RT_TMEM_COLS = 512;
constexpr uint64_t RT_DRAIN_NS = 200000000ull;     // 0.2 s for copies / MMAs in flight after an abort

struct RouterArgs {
    int64_t T;
    int K;
    int E;
    int topk;
    int chunk;                 // weight rows per TMA box and per MMA (N), a multiple of 16, <= 256
    int nchunk;                // E = chunk * nchunk
    int stages;
    int tok_pass;              // tokens per epilogue warp and pass (32 or 16)
    int norm;
    float scale;
    uint32_t a_bytes;          // x tile bytes per stage
    uint32_t stage_bytes;      // x tile + weight tile bytes per stage
    const float* bias;         // [E] or null
    int64_t* ids;              // [T, topk]
    float* weights;            // [T, topk]
    int32_t* hist;             // [gridDim.x, E + 1] or null
    int32_t* status;
    uint64_t wait_ns;          // limit of every bounded mbarrier wait (exl3_set_wait_limit_ns)
};

// 32 lanes x 16 consecutive 32-bit columns (the tail of an E that is not a multiple of 32).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// (a, ia) ranks before (b, ib): larger selection score first, then the lower expert id.
__device__ __forceinline__ bool ranks_before(float a, int ia, float b, int ib)
{
    return a > b || (a == b && ia < ib);
}

__device__ __forceinline__ float sigmoid_score(float logit)
{
    return 1.0f / (1.0f + expf(-logit));
}

// One token's routing by one warp.  `row` holds the token's sigmoid scores (shared memory), `bsel` the
// lane's bias values (expert e = lane + 32*m at index m, MPL >= E / 32 of them).  Lane l holds the
// selection scores s + bias of experts l, l + 32, ... and its own best entry in the ranks_before order;
// each of the k rounds takes the warp-wide best (butterfly arg-max over the lanes), and only the lane
// that owned it removes it and rescans.  The weights are the winners' scores over their sum (summed in
// rank order, as the oracle does) times `scale`.
template <int MPL>
__device__ __forceinline__ void select_token(const float* row, const float (&bsel)[MPL], int E, int k, int norm,
                                             float scale, int lane, int64_t* ids, float* weights, int* s_hist)
{
    float v[MPL];
    #pragma unroll
    for (int m = 0; m < MPL; ++m)
    {
        const int e = lane + 32 * m;
        v[m] = (e < E) ? row[e] + bsel[m] : -INFINITY;
    }
    float lv = -INFINITY;                            // this lane's best remaining entry
    int li = 0x7fffffff;
    #pragma unroll
    for (int m = 0; m < MPL; ++m)
        if (v[m] > -INFINITY && ranks_before(v[m], lane + 32 * m, lv, li))   // removed entries and NaN never win
        {
            lv = v[m];
            li = lane + 32 * m;
        }
    float acc = 0.0f, my_s = 0.0f;
    int my_id = -1;
    for (int j = 0; j < k; ++j)
    {
        float bv = lv;
        int bi = li;
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1)
        {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ranks_before(ov, oi, bv, bi))
            {
                bv = ov;
                bi = oi;
            }
        }
        const bool valid = bi != 0x7fffffff;        // fewer than k finite scores (NaN logits)
        if (valid && li == bi)                      // the owner removes the winner and rescans
        {
            lv = -INFINITY;
            li = 0x7fffffff;
            #pragma unroll
            for (int m = 0; m < MPL; ++m)
            {
                const int e = lane + 32 * m;
                if (e == bi) v[m] = -INFINITY;
                if (v[m] > -INFINITY && ranks_before(v[m], e, lv, li))
                {
                    lv = v[m];
                    li = e;
                }
            }
        }
        const float sw = valid ? row[bi] : 0.0f;
        acc += sw;
        if (lane == j)
        {
            my_id = valid ? bi : -1;
            my_s = sw;
        }
    }
    if (lane < k)
    {
        const float w = norm ? my_s / (acc + 1e-20f) : my_s;
        ids[lane] = my_id;                           // -1: an empty slot stays unrouted
        weights[lane] = my_id >= 0 ? w * scale : 0.0f;
        atomicAdd(&s_hist[my_id >= 0 ? my_id : E], 1);
    }
}

__device__ __forceinline__ void epilogue_bar()
{
    asm volatile("bar.sync 1, %0;" :: "n"(RT_EPI_THREADS) : "memory");
}

template <int MPL>
__global__ __launch_bounds__(RT_THREADS, 1)
void router_topk_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const RouterArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_full[RT_MAX_STAGES], bar_empty[RT_MAX_STAGES];
    __shared__ uint64_t bar_done;
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_abort;
    __shared__ int s_hist[kRouterMaxExperts + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int nkb = p.K / RT_BK;
    const int64_t row0 = (int64_t) blockIdx.x * RT_BM;

    __shared__ int s_fail, s_go;
    for (int i = threadIdx.x; i <= p.E; i += RT_THREADS) s_hist[i] = 0;
    if (threadIdx.x == 0)
    {
        s_fail = 0;
        s_go = 0;
    }
    if (warp == 1)
    {
        if (lane == 0)
        {
            for (int s = 0; s < p.stages; ++s)
            {
                mbar_init(&bar_full[s], 1);
                mbar_init(&bar_empty[s], 1);
            }
            mbar_init(&bar_done, 1);
            s_abort = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&s_tmem_base, RT_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem_base;
    volatile int* abort_flag = &s_abort;

    if (warp == 0)
    {
        // ================================================================ TMA producer
        if (lane == 0)
        {
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb)
            {
                const int s = kb % p.stages;
                if (kb >= p.stages &&
                    !mbar_wait(&bar_empty[s], ((kb / p.stages) & 1u) ^ 1u, abort_flag, p.status, p.wait_ns))
                    break;
                uint8_t* a = smem + s * p.stage_bytes;
                mbar_arrive_expect_tx(&bar_full[s], p.stage_bytes);
                tma_load_2d(a, &tmap_x, kb * RT_BK, (int32_t) row0, &bar_full[s]);
                for (int c = 0; c < p.nchunk; ++c)
                    tma_load_2d(a + p.a_bytes + c * p.chunk * 128, &tmap_w, kb * RT_BK, c * p.chunk, &bar_full[s]);
                ++issued;
            }
            // copies still in flight land before the CTA's shared memory goes away (after an abort; on
            // the normal path every stage was consumed and these return at once)
            for (int kb = issued > p.stages ? issued - p.stages : 0; kb < issued; ++kb)
                mbar_drain(&bar_full[kb % p.stages], (kb / p.stages) & 1u, RT_DRAIN_NS);
        }
    }
    else if (warp == 1)
    {
        // ================================================================ MMA issuer
        if (lane == 0)
        {
            const uint32_t idesc = idesc_f16_f32(RT_BM, p.chunk);
            for (int kb = 0; kb < nkb; ++kb)
            {
                const int s = kb % p.stages;
                if (!mbar_wait(&bar_full[s], (kb / p.stages) & 1u, abort_flag, p.status, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + s * p.stage_bytes);
                const uint64_t a_desc = smem_desc_sw128(a_addr);
                for (int c = 0; c < p.nchunk; ++c)
                {
                    const uint64_t b_desc = smem_desc_sw128(a_addr + p.a_bytes + c * p.chunk * 128);
                    #pragma unroll
                    for (int kk = 0; kk < RT_BK / 16; ++kk)
                        umma_f16(tmem_base + c * p.chunk, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
                }
                umma_commit(&bar_empty[s]);
            }
            umma_commit(&bar_done);
            // every MMA issued above has completed before TMEM can be freed
            mbar_drain(&bar_done, 0, RT_DRAIN_NS);
        }
    }
    else
    {
        // ================================================================ epilogue
        // Phase 1 (warps 2..5, thread = token = TMEM lane): the sigmoid scores of the token's logits into
        // shared memory, reusing the drained TMA ring, rows padded to E + 1 floats (conflict-free stores).
        // Phase 2 (warps 2..11, warp = token): select_token.  tok_pass tokens of each TMEM quarter per pass
        // (32, or 16 when the scores of all 128 tokens would not fit).
        const bool ph1 = warp < 6;
        const int quarter = warp & 3;
        const int ew = warp - 2;                     // epilogue warp 0..9
        if (ph1 && !__all_sync(0xffffffffu, mbar_wait(&bar_done, 0, abort_flag, p.status, p.wait_ns)))
            if (lane == 0) s_fail = 1;
        epilogue_bar();
        if (threadIdx.x == 64) s_go = !s_fail && !*abort_flag;     // one decision for every epilogue warp
        epilogue_bar();
        const bool go = s_go != 0;
        if (go)
        {
            tc_fence_after();
            const int k = p.topk, E = p.E, ld = E + 1;
            float bsel[MPL];
            #pragma unroll
            for (int m = 0; m < MPL; ++m)
            {
                const int e = lane + 32 * m;
                bsel[m] = (p.bias && e < E) ? __ldg(p.bias + e) : 0.0f;
            }
            float* sc = reinterpret_cast<float*>(smem);
            for (int p0 = 0; p0 < 32; p0 += p.tok_pass)
            {
                if (ph1)
                {
                    const bool mine = lane >= p0 && lane < p0 + p.tok_pass;
                    float* my_row = sc + (quarter * p.tok_pass + lane - p0) * ld;
                    for (int c0 = 0; c0 < E; c0 += 32)
                    {
                        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c0;
                        if (E - c0 >= 32)
                        {
                            uint32_t v[32];
                            tmem_ld32(taddr, v);
                            tmem_wait_ld();
                            #pragma unroll
                            for (int i = 0; i < 32; ++i)
                            {
                                asm volatile("" : "+r"(v[i]));
                                if (mine) my_row[c0 + i] = sigmoid_score(__uint_as_float(v[i]));
                            }
                        }
                        else
                        {
                            uint32_t v[16];                  // E % 16 == 0: a 16-column tail
                            tmem_ld16(taddr, v);
                            tmem_wait_ld();
                            #pragma unroll
                            for (int i = 0; i < 16; ++i)
                            {
                                asm volatile("" : "+r"(v[i]));
                                if (mine) my_row[c0 + i] = sigmoid_score(__uint_as_float(v[i]));
                            }
                        }
                    }
                }
                epilogue_bar();
                for (int u = ew; u < 4 * p.tok_pass; u += RT_EPI_WARPS)
                {
                    const int q = u / p.tok_pass, tt = u - q * p.tok_pass;
                    const int64_t t = row0 + q * 32 + p0 + tt;
                    if (t < p.T)
                        select_token<MPL>(sc + u * ld, bsel, E, k, p.norm, p.scale, lane, p.ids + t * k,
                                          p.weights + t * k, s_hist);
                }
                epilogue_bar();                          // the rows are rewritten by the next pass
            }
        }
        // slots of this tile: every one unrouted if the tile gave up
        const int64_t n_slots = (p.T - row0 < RT_BM ? p.T - row0 : RT_BM) * p.topk;
        if (!go)
        {
            // gave up (a wait timed out): the tile's tokens stay unrouted (id -1, weight 0), so the sort
            // that follows sees ids and a histogram row (no routed slot) that agree, and stays in bounds
            for (int64_t i = threadIdx.x - 64; i < n_slots; i += RT_EPI_THREADS)
            {
                p.ids[row0 * p.topk + i] = -1;
                p.weights[row0 * p.topk + i] = 0.0f;
            }
        }
        // the tile's histogram, once every token is counted (bin E: ids outside [0, E))
        if (p.hist)
            for (int i = threadIdx.x - 64; i <= p.E; i += RT_EPI_THREADS)
                p.hist[(int64_t) blockIdx.x * (p.E + 1) + i] = go ? s_hist[i] : (i == p.E ? (int) n_slots : 0);
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        tmem_dealloc(tmem_base, RT_TMEM_COLS);
    }
}

int make_tensor_map_rows(CUtensorMap* tmap, const void* base, int64_t rows, int K, int box_rows)
{
    auto encode = trellis::get_encode_fn();
    if (!encode) return set_error("router: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t) K, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) K * 2};
    const cuuint32_t box[2] = {(cuuint32_t) RT_BK, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error("router: cuTensorMapEncodeTiled failed (%d)", (int) cr);
    return 0;
}

std::atomic<bool> g_router_attr_set[kMaxDevices] = {};

}  // namespace

int router_chunking(int E, int* chunk, int* nchunk)
{
    if (E < 16 || E > kRouterMaxExperts || E % 16 != 0) return -1;
    const int n = (E + 255) / 256;
    if (E % (16 * n) != 0) return -1;
    *nchunk = n;
    *chunk = E / n;
    return 0;
}

int64_t router_tiles(int64_t T) { return (T + RT_BM - 1) / RT_BM; }

int launch_router_topk(const void* x, int64_t T, int K, const void* w, int E, const float* bias, int topk, int norm,
                       float scale, int64_t* ids, float* weights, int32_t* hist, int32_t* status, cudaStream_t stream)
{
    if (T <= 0) return 0;
    int chunk = 0, nchunk = 0;
    if (router_chunking(E, &chunk, &nchunk))
        return set_error("router: E must be a multiple of 16 in [16, %d], split into equal boxes of <= 256 rows that are "
                         "multiples of 16", kRouterMaxExperts);
    if (K <= 0 || K % RT_BK != 0) return set_error("router: hidden size must be a positive multiple of %d", RT_BK);
    if (topk < 1 || topk > kRouterMaxTopk || topk > E) return set_error("router: topk must be 1..%d and <= E", kRouterMaxTopk);
    RouterArgs p{};
    p.T = T; p.K = K; p.E = E; p.topk = topk; p.chunk = chunk; p.nchunk = nchunk; p.norm = norm; p.scale = scale;
    p.a_bytes = RT_BM * RT_BK * 2;
    p.stage_bytes = p.a_bytes + (uint32_t) E * RT_BK * 2;
    const uint32_t budget = 232448 - 8192;        // dynamic shared memory left beside the static arrays
    p.stages = (int) ((budget - 1024) / p.stage_bytes);
    if (p.stages > RT_MAX_STAGES) p.stages = RT_MAX_STAGES;
    if (p.stages < 2) return set_error("router: E too large for two pipeline stages");
    // the epilogue's score rows (4 warps x tok_pass tokens x (E + 1) floats) reuse the ring
    const uint32_t ring = (uint32_t) p.stages * p.stage_bytes;
    p.tok_pass = 32;
    while (p.tok_pass > 1 && 4u * p.tok_pass * (E + 1) * 4u > ring) p.tok_pass /= 2;
    p.bias = bias; p.ids = ids; p.weights = weights; p.hist = hist; p.status = status;
    p.wait_ns = wait_limit_ns();
    CUtensorMap tx, tw;
    int rc = make_tensor_map_rows(&tx, x, T, K, RT_BM);
    if (rc) return rc;
    rc = make_tensor_map_rows(&tw, w, E, K, chunk);
    if (rc) return rc;
    const size_t smem = (size_t) p.stages * p.stage_bytes + 1024;
    rc = once_per_device(g_router_attr_set, "router", [](int) {
        const void* fns[] = {(const void*) router_topk_kernel<2>, (const void*) router_topk_kernel<4>,
                             (const void*) router_topk_kernel<9>, (const void*) router_topk_kernel<16>};
        for (const void* fn : fns)
        {
            const cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 8192);
            if (err != cudaSuccess) return set_cuda_error("router: cudaFuncSetAttribute", err);
        }
        return 0;
    });
    if (rc) return rc;
    // experts per lane in the selection: the smallest instantiation holding ceil(E / 32)
    const unsigned grid = (unsigned) router_tiles(T);
    if (E <= 64) router_topk_kernel<2><<<grid, RT_THREADS, smem, stream>>>(tx, tw, p);
    else if (E <= 128) router_topk_kernel<4><<<grid, RT_THREADS, smem, stream>>>(tx, tw, p);
    else if (E <= 288) router_topk_kernel<9><<<grid, RT_THREADS, smem, stream>>>(tx, tw, p);
    else router_topk_kernel<16><<<grid, RT_THREADS, smem, stream>>>(tx, tw, p);
    return check_launch("router_topk");
}

}  // namespace exl3b
