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
//   warps 2..5  epilogue, one thread per token (TMEM lane): logits 32 columns at a time, sigmoid, bias,
//               a register top-k ordered by (selection score descending, expert id ascending), the
//               weights, and the tile's expert histogram (the route sort's first pass) in shared memory.
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
constexpr int RT_THREADS = 192;
constexpr int RT_MAX_STAGES = 6;
constexpr uint32_t RT_TMEM_COLS = 512;
constexpr uint64_t RT_WAIT_NS = 2000000000ull;     // 2 s: far above any legitimate wait
constexpr uint64_t RT_DRAIN_NS = 200000000ull;     // 0.2 s for copies / MMAs in flight after an abort

struct RouterArgs {
    int64_t T;
    int K;
    int E;
    int topk;
    int chunk;                 // weight rows per TMA box and per MMA (N), a multiple of 16, <= 256
    int nchunk;                // E = chunk * nchunk
    int stages;
    int norm;
    float scale;
    uint32_t a_bytes;          // x tile bytes per stage
    uint32_t stage_bytes;      // x tile + weight tile bytes per stage
    const float* bias;         // [E] or null
    int64_t* ids;              // [T, topk]
    float* weights;            // [T, topk]
    int32_t* hist;             // [gridDim.x, E + 1] or null
    int32_t* status;
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

// One token's running top-k in registers (every index a compile-time constant).  The k entries sit at
// the END of the arrays, sorted by ranks_before; the first kRouterMaxTopk - k slots hold +inf sentinels
// that nothing displaces, so the k-th entry (the admission threshold) is always the last slot.
struct TopK {
    float val[kRouterMaxTopk];     // selection score s + bias
    float sco[kRouterMaxTopk];     // sigmoid score s (the weight before normalisation)
    int idx[kRouterMaxTopk];       // expert id

    __device__ __forceinline__ void init(int k)
    {
        #pragma unroll
        for (int j = 0; j < kRouterMaxTopk; ++j)
        {
            const bool real = j >= kRouterMaxTopk - k;
            val[j] = real ? -INFINITY : INFINITY;
            sco[j] = 0.0f;
            idx[j] = real ? 0x7fffffff : -1;
        }
    }

    __device__ __forceinline__ void consider(float logit, int e, const float* bias)
    {
        const float s = 1.0f / (1.0f + expf(-logit));
        const float sel = s + (bias ? __ldg(bias + e) : 0.0f);
        if (!ranks_before(sel, e, val[kRouterMaxTopk - 1], idx[kRouterMaxTopk - 1])) return;
        // insert: walk down the sorted list, carrying the displaced entry
        float cv = sel, cs = s;
        int ci = e;
        #pragma unroll
        for (int j = 0; j < kRouterMaxTopk; ++j)
        {
            if (ranks_before(cv, ci, val[j], idx[j]))
            {
                const float tv = val[j], ts = sco[j];
                const int ti = idx[j];
                val[j] = cv; sco[j] = cs; idx[j] = ci;
                cv = tv; cs = ts; ci = ti;
            }
        }
    }
};

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

    __shared__ int s_never;                        // a flag nobody raises: drain waits ignore the abort
    for (int i = threadIdx.x; i <= p.E; i += RT_THREADS) s_hist[i] = 0;
    if (threadIdx.x == 0) s_never = 0;
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
                    !mbar_wait(&bar_empty[s], ((kb / p.stages) & 1u) ^ 1u, abort_flag, p.status, RT_WAIT_NS))
                    break;
                uint8_t* a = smem + s * p.stage_bytes;
                mbar_arrive_expect_tx(&bar_full[s], p.stage_bytes);
                tma_load_2d(a, &tmap_x, kb * RT_BK, (int32_t) row0, &bar_full[s]);
                for (int c = 0; c < p.nchunk; ++c)
                    tma_load_2d(a + p.a_bytes + c * p.chunk * 128, &tmap_w, kb * RT_BK, c * p.chunk, &bar_full[s]);
                ++issued;
            }
            if (*abort_flag)
            {
                // copies still in flight land before the CTA's shared memory goes away
                volatile int* never = &s_never;
                for (int kb = issued > p.stages ? issued - p.stages : 0; kb < issued; ++kb)
                    mbar_wait(&bar_full[kb % p.stages], (kb / p.stages) & 1u, never, nullptr, RT_DRAIN_NS);
            }
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
                if (!mbar_wait(&bar_full[s], (kb / p.stages) & 1u, abort_flag, p.status, RT_WAIT_NS)) break;
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
            volatile int* never = &s_never;
            mbar_wait(&bar_done, 0, never, nullptr, *abort_flag ? RT_DRAIN_NS : RT_WAIT_NS);
        }
    }
    else
    {
        // ================================================================ epilogue: one token per thread
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int64_t t = row0 + r;
        const bool done = mbar_wait(&bar_done, 0, abort_flag, p.status, RT_WAIT_NS);
        // warp-uniform decision: tcgen05.ld needs the whole warp
        if (__all_sync(0xffffffffu, done && !*abort_flag))
        {
            tc_fence_after();
            const int k = p.topk;
            TopK top;
            top.init(k);
            for (int c0 = 0; c0 < p.E; c0 += 32)
            {
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c0;
                if (p.E - c0 >= 32)
                {
                    uint32_t v[32];
                    tmem_ld32(taddr, v);
                    tmem_wait_ld();
                    #pragma unroll
                    for (int i = 0; i < 32; ++i)
                    {
                        asm volatile("" : "+r"(v[i]));
                        top.consider(__uint_as_float(v[i]), c0 + i, p.bias);
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
                        top.consider(__uint_as_float(v[i]), c0 + i, p.bias);
                    }
                }
            }
            if (t < p.T)
            {
                constexpr int KM = kRouterMaxTopk;
                float sum = 0.0f;
                #pragma unroll
                for (int j = 0; j < KM; ++j)
                    if (j >= KM - k) sum += top.sco[j];
                const float denom = sum + 1e-20f;
                #pragma unroll
                for (int j = 0; j < KM; ++j)
                    if (j >= KM - k)
                    {
                        // fewer than k finite scores (NaN logits): the empty slots stay unrouted (-1)
                        const int e = top.idx[j];
                        const bool ok = e >= 0 && e < p.E;
                        const float w = p.norm ? top.sco[j] / denom : top.sco[j];
                        p.ids[t * k + (j - (KM - k))] = ok ? e : -1;
                        p.weights[t * k + (j - (KM - k))] = ok ? w * p.scale : 0.0f;
                        atomicAdd(&s_hist[ok ? e : p.E], 1);
                    }
            }
        }
        // the tile's histogram, once every epilogue thread has counted its token
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (p.hist && !*abort_flag)
            for (int i = r; i <= p.E; i += 128) p.hist[(int64_t) blockIdx.x * (p.E + 1) + i] = s_hist[i];
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

bool g_router_attr_set[64] = {};

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
    p.bias = bias; p.ids = ids; p.weights = weights; p.hist = hist; p.status = status;
    CUtensorMap tx, tw;
    int rc = make_tensor_map_rows(&tx, x, T, K, RT_BM);
    if (rc) return rc;
    rc = make_tensor_map_rows(&tw, w, E, K, chunk);
    if (rc) return rc;
    const size_t smem = (size_t) p.stages * p.stage_bytes + 1024;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return set_cuda_error("router: cudaGetDevice", err);
    if (dev < 0 || dev >= 64) return set_error("router: device ordinal %d out of range", dev);
    if (!g_router_attr_set[dev])
    {
        err = cudaFuncSetAttribute(router_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 8192);
        if (err != cudaSuccess) return set_cuda_error("router: cudaFuncSetAttribute", err);
        g_router_attr_set[dev] = true;
    }
    router_topk_kernel<<<(unsigned) router_tiles(T), RT_THREADS, smem, stream>>>(tx, tw, p);
    return check_launch("router_topk");
}

}  // namespace exl3b
