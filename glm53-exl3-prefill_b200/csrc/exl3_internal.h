// exl3_internal.h — host-side declarations shared by the kernel translation units and the C-ABI layer.
#pragma once

#include <atomic>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

namespace exl3b {

constexpr int kMaxExperts = 1024;   // kernel/exl3_grouped_prefill.cu:44 (MAX_EXPERTS)
constexpr int kMaxDevices = 64;

// Error reporting (capi.cu): set the thread-local message returned by exl3_last_error().
int set_error(const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t err);
int check_launch(const char* what);          // cudaPeekAtLastError after a launch

// Per-device properties, cached (capi.cu).
int device_sm_count();

// Time limit of the bounded mbarrier waits in the tcgen05 kernels (capi.cu, exl3_set_wait_limit_ns).
uint64_t wait_limit_ns();

// One lock for every kernel's per-device set-up (capi.cu).
std::mutex& setup_mutex();

// Runs init(dev) once for the current device, under setup_mutex(), so that host threads starting on
// one device at the same time neither race on `done` nor run the set-up twice.  A failed init is
// retried by the next call.  Returns init's code (0 = set up).
template <class F>
int once_per_device(std::atomic<bool> (&done)[kMaxDevices], const char* what, F&& init)
{
    int dev = 0;
    const cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return set_cuda_error(what, err);
    if (dev < 0 || dev >= kMaxDevices) return set_error("%s: device ordinal %d out of range", what, dev);
    if (done[dev].load(std::memory_order_acquire)) return 0;
    std::lock_guard<std::mutex> lock(setup_mutex());
    if (done[dev].load(std::memory_order_relaxed)) return 0;
    const int rc = init(dev);
    if (rc == 0) done[dev].store(true, std::memory_order_release);
    return rc;
}

// ---- route.cu
int launch_route_sort(const void* ids, int ids_i64, const void* weights, int wdtype, int64_t T, int topk,
                      int n_experts, int max_blocks, int64_t* token_sorted, void* weight_sorted,
                      int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0, int32_t* block_expert,
                      int32_t* block_row0, int32_t* meta, int32_t* invalid_count, int32_t* scratch,
                      cudaStream_t stream);
int64_t route_sort_scratch_elems(int64_t R, int n_experts);
// Allocation-free variant: scratch in a file-scope device array of kRouteStaticScratchElems int32.
constexpr int64_t kRouteStaticScratchElems = 65536;
int launch_route_sort_noalloc(const void* ids, int ids_i64, const void* weights, int wdtype, int64_t T, int topk,
                              int n_experts, int max_blocks, int64_t* token_sorted, void* weight_sorted,
                              int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0, int32_t* block_expert,
                              int32_t* block_row0, int32_t* meta, int32_t* invalid_count, cudaStream_t stream);
int launch_build_blocks(const int32_t* counts, int n_experts, int32_t* block_expert, int32_t* block_row0,
                        int max_blocks, int32_t* meta, cudaStream_t stream);
// Router front-end (router.cu) followed by the sort's scatter pass over its output (route.cu).
int64_t route_front_scratch_elems(int64_t T, int topk, int n_experts);
int launch_route_front(const void* x, int64_t T, int K, const void* w_router, int n_experts, const float* bias,
                       int topk, int norm, float scale, int64_t* ids, float* weights, int max_blocks,
                       int64_t* token_sorted, void* weight_sorted, int32_t* expert_of_row, int32_t* counts,
                       int32_t* expert_row0, int32_t* block_expert, int32_t* block_row0, int32_t* meta,
                       int32_t* scratch, int32_t* status, cudaStream_t stream, int slot_rows = 0);

// ---- router.cu
constexpr int kRouterMaxExperts = 512;   // TMEM columns of one 128-lane accumulator
constexpr int kRouterMaxTopk = 16;
int router_chunking(int n_experts, int* chunk, int* nchunk);      // 0 if n_experts is supported
int64_t router_tiles(int64_t T);                                   // 128-token tiles (CTAs, histogram rows)
int launch_router_topk(const void* x, int64_t T, int K, const void* w_router, int n_experts, const float* bias,
                       int topk, int norm, float scale, int64_t* ids, float* weights, int32_t* hist, int32_t* status,
                       cudaStream_t stream);

// Expert parallelism: one buffer per rank, mapped into this process (CUDA IPC).  A global index g
// addresses row q = g / index_div, which is row q % rows_per_rank of rank q / rows_per_rank's buffer.
// Passed by value to kernels.
constexpr int kMaxRanks = 8;
struct PeerRows {
    const void* ptr[kMaxRanks];
    int64_t rows_per_rank;
    int64_t index_div;
};

#ifdef __CUDACC__
// Base pointer of rank `rk` by an unrolled select: a runtime index into the parameter array would copy
// it to local memory.
__device__ __forceinline__ const void* peer_ptr(const PeerRows& t, int64_t rk)
{
    const void* p = t.ptr[0];
    #pragma unroll
    for (int i = 1; i < kMaxRanks; ++i)
        if (rk == i) p = t.ptr[i];
    return p;
}
#endif

// ---- hadamard.cu
int launch_row_had(const void* src, void* dst, int64_t rows, int K, const int64_t* token_sorted,
                   const int32_t* expert_of_row, const void* suh, int64_t suh_stride, int gather,
                   cudaStream_t stream);
// rows_dev (nullable): a device int32 count; the kernels then process min(rows, *rows_dev) rows (a count
// known on the device only, such as a sort's meta[1]), with the grid sized for `rows`.
int launch_ep_row_had(const PeerRows& peers, void* dst, int64_t rows, int K, const int64_t* token_sorted,
                      const int32_t* expert_of_row, int expert_base, const void* suh, int64_t suh_stride,
                      int32_t* slot_row, const int32_t* rows_dev, cudaStream_t stream);
int launch_act_had(const void* gu, void* act, int64_t rows, int I, const int32_t* expert_of_row, int expert_base,
                   const void* suh, int64_t suh_stride, float limit, cudaStream_t stream,
                   const int32_t* rows_dev = nullptr);
int launch_ep_pull_rows(const PeerRows& x, int n_ranks, int rank, int K, const int64_t* ids, int topk, int64_t e0,
                        int64_t e1, void* x_pulled, cudaStream_t stream);
int launch_ep_combine_push(const float* y, int K, const int64_t* ids, int topk, int64_t e0, int64_t e1,
                           const int32_t* slot_row, const PeerRows& staging, int n_ranks, int rank, int f16,
                           cudaStream_t stream);
int launch_ep_combine_reduce(const void* staging, int f16, const int64_t* ids, int64_t T, int topk, int n_experts,
                             int n_ranks, float* out, int K, cudaStream_t stream);
int launch_combine_slots(const float* y, const void* ids, int ids_i64, int64_t T, int topk, int n_experts, float* out,
                         int K, int accumulate, cudaStream_t stream);

// ---- trellis_gemm.cu
enum GemmMode : int {
    kModeStoreF16 = 0,     // out fp16 [rows, *]: row store (gate|up stage)
    kModeScatterAtomic = 1,// out fp32 [T, *] += w[r] * y via atomics (down stage)
    kModeStoreF32 = 2,     // out fp32 [rows, *]: row store (fat_gemm_v2)
    kModeScatterAdd = 3,   // out fp32 [T, *] += w[r] * y, non-atomic (fat_gemm_v2_scatter)
    kModeStoreWeighted = 4,// out fp32 [rows, *] = w[r] * y: row store of the weighted rows (expert parallelism)
    kModeStoreRows = 5,    // out fp32 [*, *]: row token_sorted[r] = w[r] * y (each destination row once)
};

struct GemmProblem {
    const void* a;                 // fp16 [a_rows, size_k], row-major, 16-byte aligned
    int64_t a_rows;
    int size_k;
    const void* packed[2];         // int16 [E, tiles_k, tiles_n, 64] views (gate, up) or (w, null)
    int64_t expert_stride_words;
    int tiles_n;                   // trellis tiles along N of each source matrix
    const void* svh[2];            // fp16 [E, N] views
    int64_t svh_stride;
    const int32_t* counts;         // [E] (device) or null: one expert with single_count rows
    const int32_t* expert_row0;    // [E] (device) or null
    int n_experts;
    int single_count;
    const int64_t* token_sorted;   // [rows] (modes 1, 3)
    const void* route_weight;      // fp16 [rows] (modes 1, 3), null = weight 1
    void* out;
    int64_t out_ld;                // output row stride in elements
    int mode;
    int gate_up;                   // 1: two source matrices written side by side (mode 0)
    int32_t* status;               // device error word (may be null)
};

int launch_trellis_gemm(const GemmProblem& p, cudaStream_t stream);
int trellis_gemm_smem_bytes();

}  // namespace exl3b
