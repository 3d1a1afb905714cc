// capi.cu — the extern "C" boundary of libexl3_b200.so (declared in include/exl3_b200.h).
//
// Validates sizes, alignment and codes the way the reference's TORCH_CHECKs do
// (kernel/exl3_grouped_prefill.cu:288-371, kernel/exl3_fat_gemm_v2.cu:236-252), then forwards to
// the kernel launchers.  Errors are returned as codes with a thread-local message.  Apart from the
// expert-parallel buffer functions (exl3_ep_alloc / exl3_ep_ipc_open), nothing here allocates device
// memory or synchronises the host.
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <string>

#include <cuda_runtime.h>

#include "exl3_internal.h"
#include "../../include/exl3_b200.h"

namespace exl3b {

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_sm_count[kMaxDevices] = {};
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;         // 2 s
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};
}

std::mutex& setup_mutex()
{
    static std::mutex mu;
    return mu;
}

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int set_error(const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return EXL3_E_INVALID;
}

int set_cuda_error(const char* what, cudaError_t err)
{
    char buf[512];
    snprintf(buf, sizeof(buf), "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
    g_last_error = buf;
    return EXL3_E_CUDA;
}

int check_launch(const char* what)
{
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return set_cuda_error(what, err);
    return EXL3_OK;
}

int device_sm_count()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < kMaxDevices)
    {
        const int cached = g_sm_count[dev].load(std::memory_order_relaxed);
        if (cached > 0) return cached;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0 && dev < kMaxDevices) g_sm_count[dev].store(n, std::memory_order_relaxed);
    return n;
}

}  // namespace exl3b

using namespace exl3b;

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_fat_common(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed, int64_t size_n,
                     const void* out, const void* svh, int64_t K, int mcg, int mul1, int64_t variant)
{
    if (!a || !packed || !out || !svh) return set_error("tensors must be CUDA");
    if (K != 4 || !mcg || mul1) return set_error("only K4 MCG tensors");
    if (size_n % 128 != 0) return set_error("N must be divisible by 128");
    if (size_k % 64 != 0) return set_error("K must be divisible by 64");
    if (size_m < 0) return set_error("a must have a non-negative number of rows");
    if (variant < 0 || variant > 3) return set_error("unknown variant");
    if (!aligned16(a) || !aligned16(packed) || !aligned16(out) || !aligned16(svh))
        return set_error("tensors must be 16-byte aligned");
    return EXL3_OK;
}

}  // namespace

extern "C" {

const char* exl3_last_error(void) { return g_last_error.c_str(); }

int exl3_abi_version(void) { return EXL3_B200_ABI_VERSION; }

int64_t exl3_set_wait_limit_ns(int64_t ns)
{
    const uint64_t v = ns < 0 ? kDefaultWaitLimitNs : (uint64_t) ns;
    return (int64_t) g_wait_limit_ns.exchange(v, std::memory_order_relaxed);
}

int exl3_build_blocks(const int32_t* counts, int64_t n_experts, int32_t* block_expert, int32_t* block_row0,
                      int64_t max_blocks, int32_t* meta, void* stream)
{
    if (n_experts > kMaxExperts) return set_error("too many experts");
    if (n_experts < 0 || max_blocks < 0 || max_blocks > 0x7fffffff) return set_error("invalid sizes");
    if ((n_experts > 0 && !counts) || (max_blocks > 0 && (!block_expert || !block_row0)) || !meta)
        return set_error("int32 tensors");
    return launch_build_blocks(counts, (int) n_experts, block_expert, block_row0, (int) max_blocks, meta,
                               as_stream(stream));
}

int exl3_route_sort(const void* ids, int ids_is_int64, const void* weights, int weight_dtype, int64_t T,
                    int64_t topk, int64_t n_experts, int64_t max_blocks, int64_t* token_sorted,
                    void* weight_sorted, int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0,
                    int32_t* block_expert, int32_t* block_row0, int32_t* meta, int32_t* invalid_count,
                    int32_t* scratch, int64_t scratch_elems, void* stream)
{
    if (n_experts <= 0 || n_experts > kMaxExperts) return set_error("too many experts");
    if (T >= 0 && topk > 0 && (!scratch || scratch_elems < route_sort_scratch_elems(T * topk, (int) n_experts)))
        return set_error("route_sort: scratch must hold exl3_route_sort_scratch_elems() int32 values");
    if (T < 0 || topk <= 0 || T * topk > 0x7fffffffLL) return set_error("invalid routing shape");
    if (weight_dtype < EXL3_DTYPE_F32 || weight_dtype > EXL3_DTYPE_BF16) return set_error("unknown weight dtype");
    if (max_blocks < 0 || max_blocks > 0x7fffffffLL) return set_error("invalid max_blocks");
    if ((T > 0 && (!ids || !weights || !token_sorted || !weight_sorted || !expert_of_row)) || !counts ||
        !expert_row0 || !meta || (max_blocks > 0 && (!block_expert || !block_row0)))
        return set_error("routing tensors must be CUDA");
    return launch_route_sort(ids, ids_is_int64 ? 1 : 0, weights, weight_dtype, T, (int) topk, (int) n_experts,
                             (int) max_blocks, token_sorted, weight_sorted, expert_of_row, counts, expert_row0,
                             block_expert, block_row0, meta, invalid_count, scratch, as_stream(stream));
}

int exl3_route_sort_noalloc(const void* ids, int ids_is_int64, const void* weights, int weight_dtype, int64_t T,
                            int64_t topk, int64_t n_experts, int64_t max_blocks, int64_t* token_sorted,
                            void* weight_sorted, int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0,
                            int32_t* block_expert, int32_t* block_row0, int32_t* meta, int32_t* invalid_count,
                            void* stream)
{
    if (n_experts <= 0 || n_experts > kMaxExperts) return set_error("too many experts");
    if (T < 0 || topk <= 0 || T * topk > 0x7fffffffLL) return set_error("invalid routing shape");
    if (weight_dtype < EXL3_DTYPE_F32 || weight_dtype > EXL3_DTYPE_BF16) return set_error("unknown weight dtype");
    if (max_blocks < 0 || max_blocks > 0x7fffffffLL) return set_error("invalid max_blocks");
    if ((T > 0 && (!ids || !weights || !token_sorted || !weight_sorted || !expert_of_row)) || !counts ||
        !expert_row0 || !meta || (max_blocks > 0 && (!block_expert || !block_row0)))
        return set_error("routing tensors must be CUDA");
    return launch_route_sort_noalloc(ids, ids_is_int64 ? 1 : 0, weights, weight_dtype, T, (int) topk,
                                     (int) n_experts, (int) max_blocks, token_sorted, weight_sorted, expert_of_row,
                                     counts, expert_row0, block_expert, block_row0, meta, invalid_count,
                                     as_stream(stream));
}

int64_t exl3_route_sort_scratch_elems(int64_t rows, int64_t n_experts)
{
    if (rows < 0 || n_experts <= 0 || n_experts > kMaxExperts) return -1;
    return route_sort_scratch_elems(rows, (int) n_experts);
}

namespace {

int check_router_args(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E, int64_t topk,
                      double scale, const int64_t* ids, const float* weights)
{
    int chunk = 0, nchunk = 0;
    if (router_chunking((int) (E > 0x7fffffff ? 0 : E), &chunk, &nchunk))
        return set_error("router: E must be a multiple of 16 in [16, %d] that splits into equal boxes of at most 256 "
                         "rows, each a multiple of 16", kRouterMaxExperts);
    if (d <= 0 || d % 64 != 0 || d > 0x7fffffffLL) return set_error("router: hidden size must be a positive multiple of 64");
    if (topk < 1 || topk > kRouterMaxTopk || topk > E) return set_error("router: topk must be 1..%d and <= E", kRouterMaxTopk);
    if (T < 0 || T * topk > 0x7fffffffLL) return set_error("invalid routing shape");
    if (!(scale == scale) || scale > 3.0e38 || scale < -3.0e38) return set_error("router: scale must be finite");
    if (T == 0) return EXL3_OK;
    if (!x || !w_router || !ids || !weights) return set_error("tensors must be CUDA");
    if (!aligned16(x) || !aligned16(w_router)) return set_error("router: x and the router weight must be 16-byte aligned");
    return EXL3_OK;
}

}  // namespace

int exl3_router_topk(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E, const float* bias,
                     int64_t topk, int64_t norm, double scale, int64_t* ids, float* weights, int32_t* status,
                     void* stream)
{
    const int rc = check_router_args(x, T, d, w_router, E, topk, scale, ids, weights);
    if (rc || T == 0) return rc;
    return launch_router_topk(x, T, (int) d, w_router, (int) E, bias, (int) topk, norm ? 1 : 0, (float) scale, ids,
                              weights, nullptr, status, as_stream(stream));
}

int64_t exl3_route_front_scratch_elems(int64_t T, int64_t topk, int64_t E)
{
    if (T < 0 || topk < 1 || topk > kRouterMaxTopk || E <= 0 || E > kRouterMaxExperts) return -1;
    return route_front_scratch_elems(T, (int) topk, (int) E);
}

int exl3_route_front(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E, const float* bias,
                     int64_t topk, int64_t norm, double scale, int64_t* ids, float* weights, int64_t* token_sorted,
                     void* weight_sorted, int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0,
                     int32_t* block_expert, int32_t* block_row0, int64_t max_blocks, int32_t* meta, int32_t* scratch,
                     int64_t scratch_elems, int32_t* status, void* stream)
{
    int rc = check_router_args(x, T, d, w_router, E, topk, scale, ids, weights);
    if (rc) return rc;
    if (!scratch || scratch_elems < route_front_scratch_elems(T, (int) topk, (int) E))
        return set_error("route_front: scratch must hold exl3_route_front_scratch_elems() int32 values");
    if (max_blocks < 0 || max_blocks > 0x7fffffffLL) return set_error("invalid max_blocks");
    if ((T > 0 && (!token_sorted || !weight_sorted || !expert_of_row)) || !counts || !expert_row0 || !meta ||
        (max_blocks > 0 && (!block_expert || !block_row0)))
        return set_error("routing tensors must be CUDA");
    return launch_route_front(x, T, (int) d, w_router, (int) E, bias, (int) topk, norm ? 1 : 0, (float) scale, ids,
                              weights, (int) max_blocks, token_sorted, weight_sorted, expert_of_row, counts,
                              expert_row0, block_expert, block_row0, meta, scratch, status, as_stream(stream));
}

int exl3_route_front_slots(const void* x, int64_t T, int64_t d, const void* w_router, int64_t E, const float* bias,
                           int64_t topk, int64_t norm, double scale, int64_t* ids, float* weights, int64_t* slot_sorted,
                           void* weight_sorted, int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0,
                           int32_t* block_expert, int32_t* block_row0, int64_t max_blocks, int32_t* meta,
                           int32_t* scratch, int64_t scratch_elems, int32_t* status, void* stream)
{
    int rc = check_router_args(x, T, d, w_router, E, topk, scale, ids, weights);
    if (rc) return rc;
    if (!scratch || scratch_elems < route_front_scratch_elems(T, (int) topk, (int) E))
        return set_error("route_front: scratch must hold exl3_route_front_scratch_elems() int32 values");
    if (max_blocks < 0 || max_blocks > 0x7fffffffLL) return set_error("invalid max_blocks");
    if ((T > 0 && (!slot_sorted || !weight_sorted || !expert_of_row)) || !counts || !expert_row0 || !meta ||
        (max_blocks > 0 && (!block_expert || !block_row0)))
        return set_error("routing tensors must be CUDA");
    return launch_route_front(x, T, (int) d, w_router, (int) E, bias, (int) topk, norm ? 1 : 0, (float) scale, ids,
                              weights, (int) max_blocks, slot_sorted, weight_sorted, expert_of_row, counts,
                              expert_row0, block_expert, block_row0, meta, scratch, status, as_stream(stream), 1);
}

int exl3_combine_slots(const float* y, const void* ids, int ids_is_int64, int64_t T, int64_t topk, int64_t n_experts,
                       float* out, int64_t K, int accumulate, void* stream)
{
    if (T < 0 || T > 0x7fffffffLL) return set_error("invalid token count");
    if (topk < 1 || topk > 32) return set_error("combine_slots: topk must be 1..32");
    if (n_experts <= 0 || n_experts > kMaxExperts) return set_error("too many experts");
    if (K <= 0 || K % 128 != 0) return set_error("combine_slots: K must be a multiple of 128");
    if (T == 0) return EXL3_OK;
    if (!y || !ids || !out) return set_error("tensors must be CUDA");
    if (!aligned16(y) || !aligned16(out)) return set_error("combine_slots: y and out must be 16-byte aligned");
    return launch_combine_slots(y, ids, ids_is_int64 ? 1 : 0, T, (int) topk, (int) n_experts, out, (int) K,
                                accumulate ? 1 : 0, as_stream(stream));
}

int exl3_row_had(const void* src, int64_t src_rows, void* dst, int64_t rows, int64_t K,
                 const int64_t* token_sorted, const int32_t* expert_of_row, const void* suh,
                 int64_t suh_stride, int gather, void* stream)
{
    if (K <= 0 || K % 128 != 0) return set_error("K must be a multiple of 128 and match suh");
    if (rows < 0 || src_rows < 0 || rows > 0x7fffffffLL) return set_error("invalid row count");
    if (!gather && src_rows < rows) return set_error("src must have at least `rows` rows");
    if (rows == 0) return EXL3_OK;
    if (!src || !dst || !expert_of_row || !suh || (gather && !token_sorted)) return set_error("tensors must be CUDA");
    if (!aligned16(src) || !aligned16(dst) || !aligned16(suh) || (suh_stride % 8) != 0)
        return set_error("row_had: fp16 tensors must be 16-byte aligned (suh row stride a multiple of 8)");
    return launch_row_had(src, dst, rows, (int) K, token_sorted, expert_of_row, suh, suh_stride, gather,
                          as_stream(stream));
}

int exl3_act_had(const void* gu, void* act, int64_t rows, int64_t I, const int32_t* expert_of_row,
                 const void* suh_down, int64_t suh_stride, double limit, void* stream)
{
    if (I <= 0 || I % 128 != 0) return set_error("gate|up width must be 2I, I multiple of 128");
    if (rows < 0 || rows > 0x7fffffffLL) return set_error("invalid row count");
    if (rows == 0) return EXL3_OK;
    if (!gu || !act || !expert_of_row || !suh_down) return set_error("tensors must be CUDA");
    if (!aligned16(gu) || !aligned16(act) || !aligned16(suh_down) || (suh_stride % 8) != 0)
        return set_error("act_had: fp16 tensors must be 16-byte aligned (suh row stride a multiple of 8)");
    return launch_act_had(gu, act, rows, (int) I, expert_of_row, 0, suh_down, suh_stride, (float) limit,
                          as_stream(stream));
}

int exl3_grouped_gemm(const void* a, int64_t rows, int64_t size_k, const int16_t* packed_gate,
                      const int16_t* packed_up, int64_t n_experts, int64_t tiles_k, int64_t tiles_n,
                      int64_t expert_stride_words, const void* svh_gate, const void* svh_up,
                      int64_t svh_stride, const int32_t* block_expert, const int32_t* block_row0,
                      int64_t max_blocks, const int32_t* counts, const int32_t* expert_row0,
                      const int64_t* token_sorted, const void* route_weight, void* out, int64_t out_rows,
                      int64_t out_cols, int64_t mode, int32_t* status, void* stream)
{
    (void) block_expert; (void) block_row0; (void) max_blocks;
    if (size_k != tiles_k * 16 || size_k % 64 != 0) return set_error("K mismatch");
    const int64_t size_n_each = tiles_n * 16;
    if (size_n_each <= 0 || size_n_each % 128 != 0) return set_error("N must be a multiple of 128");
    if (n_experts <= 0 || n_experts > kMaxExperts) return set_error("too many experts");
    if (!counts || !expert_row0) return set_error("counts / expert_row0 must be CUDA");
    const int n_tensors = packed_up ? 2 : 1;
    if (packed_up && !svh_up) return set_error("gate/up strides must match");
    if (expert_stride_words < tiles_k * tiles_n * 64) return set_error("packed expert stride too small");
    if (svh_stride < size_n_each) return set_error("svh N mismatch");
    GemmProblem p{};
    p.a = a; p.a_rows = rows; p.size_k = (int) size_k;
    p.packed[0] = packed_gate; p.packed[1] = packed_up;
    p.expert_stride_words = expert_stride_words; p.tiles_n = (int) tiles_n;
    p.svh[0] = svh_gate; p.svh[1] = svh_up; p.svh_stride = svh_stride;
    p.counts = counts; p.expert_row0 = expert_row0; p.n_experts = (int) n_experts; p.single_count = 0;
    p.status = status;
    if (mode == 0)
    {
        if (out_cols != n_tensors * size_n_each) return set_error("mode 0: out fp16 [rows, n_tensors*N]");
        p.mode = kModeStoreF16; p.gate_up = n_tensors == 2 ? 1 : 0;
        p.out = out; p.out_ld = out_cols;
    }
    else if (mode == 1)
    {
        if (out_cols != size_n_each || n_tensors != 1) return set_error("mode 1: out fp32 [T, N], single tensor");
        if (!token_sorted || !route_weight) return set_error("routing dtypes");
        p.mode = kModeScatterAtomic; p.gate_up = 0;
        p.token_sorted = token_sorted; p.route_weight = route_weight;
        p.out = out; p.out_ld = out_cols;
        (void) out_rows;
    }
    else if (mode == 2)
    {
        if (out_cols != size_n_each || n_tensors != 1) return set_error("mode 2: out fp32 [rows, N], single tensor");
        if (!token_sorted || !route_weight) return set_error("routing dtypes");
        p.mode = kModeStoreRows; p.gate_up = 0;
        p.token_sorted = token_sorted; p.route_weight = route_weight;
        p.out = out; p.out_ld = out_cols;
    }
    else
        return set_error("mode must be 0 (gate|up), 1 (down scatter) or 2 (down row store)");
    if (rows == 0) return EXL3_OK;
    if (!a || !packed_gate || !svh_gate || !out) return set_error("tensors must be CUDA");
    return launch_trellis_gemm(p, as_stream(stream));
}

int exl3_fat_gemm_v2(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed, int64_t size_n,
                     float* out, const void* svh, int64_t K, int mcg, int mul1, int64_t variant,
                     int32_t* status, void* stream)
{
    const int rc = check_fat_common(a, size_m, size_k, packed, size_n, out, svh, K, mcg, mul1, variant);
    if (rc) return rc;
    if (size_m == 0) return EXL3_OK;
    if (size_m > 0x7fffffffLL) return set_error("too many rows");
    GemmProblem p{};
    p.a = a; p.a_rows = size_m; p.size_k = (int) size_k;
    p.packed[0] = packed; p.packed[1] = nullptr;
    p.tiles_n = (int) (size_n / 16);
    p.expert_stride_words = (size_k / 16) * (size_n / 16) * 64;
    p.svh[0] = svh; p.svh[1] = nullptr; p.svh_stride = size_n;
    p.counts = nullptr; p.expert_row0 = nullptr; p.n_experts = 1; p.single_count = (int) size_m;
    p.mode = kModeStoreF32; p.gate_up = 0;
    p.out = out; p.out_ld = size_n;
    p.status = status;
    return launch_trellis_gemm(p, as_stream(stream));
}

int exl3_fat_gemm_v2_scatter(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed,
                             int64_t size_n, float* out, int64_t out_rows, const void* svh,
                             const int64_t* token_idx, const void* route_weight, int64_t K, int mcg,
                             int mul1, int64_t variant, int32_t* status, void* stream)
{
    const int rc = check_fat_common(a, size_m, size_k, packed, size_n, out, svh, K, mcg, mul1, variant);
    if (rc) return rc;
    if (size_m == 0) return EXL3_OK;
    if (!token_idx || !route_weight) return set_error("routing tensors");
    if (size_m > 0x7fffffffLL) return set_error("too many rows");
    (void) out_rows;
    GemmProblem p{};
    p.a = a; p.a_rows = size_m; p.size_k = (int) size_k;
    p.packed[0] = packed; p.packed[1] = nullptr;
    p.tiles_n = (int) (size_n / 16);
    p.expert_stride_words = (size_k / 16) * (size_n / 16) * 64;
    p.svh[0] = svh; p.svh[1] = nullptr; p.svh_stride = size_n;
    p.counts = nullptr; p.expert_row0 = nullptr; p.n_experts = 1; p.single_count = (int) size_m;
    p.token_sorted = token_idx; p.route_weight = route_weight;
    p.mode = kModeScatterAdd; p.gate_up = 0;
    p.out = out; p.out_ld = size_n;
    p.status = status;
    return launch_trellis_gemm(p, as_stream(stream));
}

int64_t exl3_smem_bytes(int64_t variant)
{
    if (variant < 0 || variant > 3) return -1;
    return trellis_gemm_smem_bytes();
}

int exl3_fat_gemm(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed, int64_t size_n,
                  float* out, const void* svh, int64_t K, int mcg, int mul1, int32_t* status, void* stream)
{
    return exl3_fat_gemm_v2(a, size_m, size_k, packed, size_n, out, svh, K, mcg, mul1, 0, status, stream);
}

int exl3_fat_gemm_scatter(const void* a, int64_t size_m, int64_t size_k, const int16_t* packed,
                          int64_t size_n, float* out, int64_t out_rows, const void* svh,
                          const int64_t* token_idx, const void* route_weight, int64_t K, int mcg, int mul1,
                          int32_t* status, void* stream)
{
    return exl3_fat_gemm_v2_scatter(a, size_m, size_k, packed, size_n, out, out_rows, svh, token_idx,
                                    route_weight, K, mcg, mul1, 0, status, stream);
}

// ------------------------------------------------------------------------------------ expert parallelism
int exl3_ep_alloc(int64_t bytes, void** ptr)
{
    if (!ptr || bytes <= 0) return set_error("ep_alloc: invalid arguments");
    *ptr = nullptr;
    const cudaError_t err = cudaMalloc(ptr, (size_t) bytes);
    if (err != cudaSuccess) return set_cuda_error("ep_alloc: cudaMalloc", err);
    return EXL3_OK;
}

int exl3_ep_free(void* ptr)
{
    if (!ptr) return EXL3_OK;
    const cudaError_t err = cudaFree(ptr);
    if (err != cudaSuccess) return set_cuda_error("ep_free: cudaFree", err);
    return EXL3_OK;
}

int exl3_ep_ipc_handle(const void* ptr, void* handle)
{
    if (!ptr || !handle) return set_error("ep_ipc_handle: invalid arguments");
    cudaIpcMemHandle_t h;
    const cudaError_t err = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (err != cudaSuccess) return set_cuda_error("ep_ipc_handle: cudaIpcGetMemHandle", err);
    static_assert(sizeof(h) == EXL3_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return EXL3_OK;
}

int exl3_ep_ipc_open(const void* handle, void** ptr)
{
    if (!ptr || !handle) return set_error("ep_ipc_open: invalid arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return set_cuda_error("ep_ipc_open: cudaIpcOpenMemHandle", err);
    return EXL3_OK;
}

int exl3_ep_ipc_close(void* ptr)
{
    if (!ptr) return EXL3_OK;
    const cudaError_t err = cudaIpcCloseMemHandle(ptr);
    if (err != cudaSuccess) return set_cuda_error("ep_ipc_close: cudaIpcCloseMemHandle", err);
    return EXL3_OK;
}

namespace {

int make_peer_table(const void* const* ptrs, int64_t n_ranks, int64_t rows_per_rank, int64_t index_div, PeerRows* t)
{
    if (!ptrs || n_ranks < 1 || n_ranks > kMaxRanks) return set_error("ep: 1..%d ranks", kMaxRanks);
    if (rows_per_rank <= 0 || rows_per_rank > 0x7fffffffLL) return set_error("ep: invalid rows per rank");
    if (index_div <= 0 || index_div > 32) return set_error("ep: topk must be 1..32");
    *t = PeerRows{};
    for (int64_t i = 0; i < n_ranks; ++i)
    {
        if (!ptrs[i] || !aligned16(ptrs[i])) return set_error("ep: rank %d buffer must be a 16-byte aligned CUDA pointer", (int) i);
        t->ptr[i] = ptrs[i];
    }
    t->rows_per_rank = rows_per_rank;
    t->index_div = index_div;
    return EXL3_OK;
}

}  // namespace

int exl3_ep_pull_rows(const void* const* x_ranks, int64_t n_ranks, int64_t rank, int64_t tokens_per_rank, int64_t K,
                      const int64_t* ids_pos, int64_t topk, int64_t e0, int64_t e1, void* x_pulled, void* stream)
{
    if (K <= 0 || K % 128 != 0) return set_error("K must be a multiple of 128");
    PeerRows x;
    const int rc = make_peer_table(x_ranks, n_ranks, tokens_per_rank, topk, &x);
    if (rc) return rc;
    if (rank < 0 || rank >= n_ranks) return set_error("ep: rank outside [0, n_ranks)");
    if (e0 < 0 || e1 <= e0 || e1 > kMaxExperts) return set_error("ep: invalid expert range");
    if (n_ranks == 1) return EXL3_OK;                     // nothing lives on another GPU
    if (!ids_pos || !x_pulled) return set_error("tensors must be CUDA");
    if (!aligned16(x_pulled)) return set_error("ep_pull_rows: x_pulled must be 16-byte aligned");
    return launch_ep_pull_rows(x, (int) n_ranks, (int) rank, (int) K, ids_pos, (int) topk, e0, e1, x_pulled,
                               as_stream(stream));
}

int exl3_ep_row_had(const void* const* x_ranks, int64_t n_ranks, int64_t tokens_per_rank, int64_t topk, void* dst,
                    int64_t rows, int64_t K, const int64_t* slot_sorted, const int32_t* expert_of_row,
                    int64_t expert_base, const void* suh, int64_t suh_stride, int32_t* slot_row,
                    const int32_t* rows_dev, void* stream)
{
    if (K <= 0 || K % 128 != 0) return set_error("K must be a multiple of 128 and match suh");
    if (rows < 0 || rows > 0x7fffffffLL) return set_error("invalid row count");
    if (expert_base < 0 || expert_base > kMaxExperts) return set_error("ep_row_had: invalid expert_base");
    PeerRows peers;
    const int rc = make_peer_table(x_ranks, n_ranks, tokens_per_rank, topk, &peers);
    if (rc) return rc;
    if (rows == 0) return EXL3_OK;
    if (!dst || !slot_sorted || !expert_of_row || !suh) return set_error("tensors must be CUDA");
    if (!aligned16(dst) || !aligned16(suh) || (suh_stride % 8) != 0)
        return set_error("row_had: fp16 tensors must be 16-byte aligned (suh row stride a multiple of 8)");
    return launch_ep_row_had(peers, dst, rows, (int) K, slot_sorted, expert_of_row, (int) expert_base, suh,
                             suh_stride, slot_row, rows_dev, as_stream(stream));
}

int exl3_ep_act_had(const void* gu, void* act, int64_t rows, int64_t I, const int32_t* expert_of_row,
                    int64_t expert_base, const void* suh_down, int64_t suh_stride, double limit,
                    const int32_t* rows_dev, void* stream)
{
    if (I <= 0 || I % 128 != 0) return set_error("gate|up width must be 2I, I multiple of 128");
    if (rows < 0 || rows > 0x7fffffffLL) return set_error("invalid row count");
    if (expert_base < 0 || expert_base > kMaxExperts) return set_error("ep_act_had: invalid expert_base");
    if (rows == 0) return EXL3_OK;
    if (!gu || !act || !expert_of_row || !suh_down) return set_error("tensors must be CUDA");
    if (!aligned16(gu) || !aligned16(act) || !aligned16(suh_down) || (suh_stride % 8) != 0)
        return set_error("act_had: fp16 tensors must be 16-byte aligned (suh row stride a multiple of 8)");
    return launch_act_had(gu, act, rows, (int) I, expert_of_row, (int) expert_base, suh_down, suh_stride,
                          (float) limit, as_stream(stream), rows_dev);
}

int exl3_ep_gemm_store(const void* a, int64_t rows, int64_t size_k, const int16_t* packed, int64_t n_experts,
                       int64_t tiles_k, int64_t tiles_n, int64_t expert_stride_words, const void* svh,
                       int64_t svh_stride, const int32_t* counts, const int32_t* expert_row0, const void* route_weight,
                       float* y_local, int32_t* status, void* stream)
{
    if (size_k != tiles_k * 16 || size_k % 64 != 0) return set_error("K mismatch");
    const int64_t size_n = tiles_n * 16;
    if (size_n <= 0 || size_n % 128 != 0) return set_error("N must be a multiple of 128");
    if (n_experts <= 0 || n_experts > kMaxExperts) return set_error("too many experts");
    if (!counts || !expert_row0) return set_error("counts / expert_row0 must be CUDA");
    if (expert_stride_words < tiles_k * tiles_n * 64) return set_error("packed expert stride too small");
    if (svh_stride < size_n) return set_error("svh N mismatch");
    if (rows < 0 || rows > 0x7fffffffLL) return set_error("invalid row count");
    if (rows == 0) return EXL3_OK;
    if (!a || !packed || !svh || !route_weight || !y_local) return set_error("tensors must be CUDA");
    if (!aligned16(y_local)) return set_error("ep_gemm_store: y_local must be 16-byte aligned");
    GemmProblem p{};
    p.a = a; p.a_rows = rows; p.size_k = (int) size_k;
    p.packed[0] = packed; p.packed[1] = nullptr;
    p.expert_stride_words = expert_stride_words; p.tiles_n = (int) tiles_n;
    p.svh[0] = svh; p.svh[1] = nullptr; p.svh_stride = svh_stride;
    p.counts = counts; p.expert_row0 = expert_row0; p.n_experts = (int) n_experts; p.single_count = 0;
    p.token_sorted = nullptr; p.route_weight = route_weight;
    p.mode = kModeStoreWeighted; p.gate_up = 0;
    p.out = y_local; p.out_ld = size_n;
    p.status = status;
    return launch_trellis_gemm(p, as_stream(stream));
}

int exl3_ep_combine_push(const float* y_local, int64_t K, const int64_t* ids_pos, int64_t topk, int64_t e0,
                         int64_t e1, const int32_t* slot_row, void* const* staging_ranks, int64_t n_ranks,
                         int64_t rank, int64_t tokens_per_rank, int64_t staging_f16, void* stream)
{
    if (K <= 0 || K % 128 != 0) return set_error("K must be a multiple of 128");
    PeerRows staging;
    const int rc = make_peer_table(const_cast<const void* const*>(staging_ranks), n_ranks, tokens_per_rank, topk,
                                   &staging);
    if (rc) return rc;
    if (rank < 0 || rank >= n_ranks) return set_error("ep: rank outside [0, n_ranks)");
    if (e0 < 0 || e1 <= e0 || e1 > kMaxExperts) return set_error("ep: invalid expert range");
    if (staging_f16 != 0 && staging_f16 != 1) return set_error("ep: staging_f16 must be 0 or 1");
    if (!y_local || !ids_pos || !slot_row) return set_error("tensors must be CUDA");
    if (!aligned16(y_local)) return set_error("ep_combine_push: y_local must be 16-byte aligned");
    return launch_ep_combine_push(y_local, (int) K, ids_pos, (int) topk, e0, e1, slot_row, staging, (int) n_ranks,
                                  (int) rank, (int) staging_f16, as_stream(stream));
}

int exl3_ep_combine_reduce(const void* staging, int64_t staging_f16, const int64_t* ids_pos, int64_t T, int64_t topk,
                           int64_t n_experts, int64_t n_ranks, float* out, int64_t K, void* stream)
{
    if (T < 0 || T > 0x7fffffffLL) return set_error("invalid token count");
    if (topk < 1 || topk > 32) return set_error("ep: topk must be 1..32");
    if (n_experts <= 0 || n_experts > kMaxExperts) return set_error("too many experts");
    if (n_ranks < 1 || n_ranks > kMaxRanks || n_ranks > n_experts) return set_error("ep: 1..%d ranks", kMaxRanks);
    if (K <= 0 || K % 128 != 0) return set_error("ep_combine_reduce: K must be a multiple of 128");
    if (staging_f16 != 0 && staging_f16 != 1) return set_error("ep: staging_f16 must be 0 or 1");
    if (T == 0) return EXL3_OK;
    if (!staging || !ids_pos || !out) return set_error("tensors must be CUDA");
    if (!aligned16(staging) || !aligned16(out)) return set_error("ep_combine_reduce: buffers must be 16-byte aligned");
    return launch_ep_combine_reduce(staging, (int) staging_f16, ids_pos, T, (int) topk, (int) n_experts, (int) n_ranks,
                                    out, (int) K, as_stream(stream));
}

}  // extern "C"
