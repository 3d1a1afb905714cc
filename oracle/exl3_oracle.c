/*
 * exl3_oracle.c — CPU restatement of the routed-expert EXL3 MoE prefill path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the GPU kernels are compared against; the
 * product never links, loads or calls it.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm use it.
 *
 * What is restated, and from where (paths are within the reference project):
 *   - fp16 rounding points: kernel/exl3_grouped_prefill.cu:114 (row_had writes fp16), :136 (act is
 *     rounded to fp16 before its Hadamard), :140 (act_had writes fp16), :273 (gate|up written fp16),
 *     :275 (down projection scattered in fp32).
 *   - H128: Sylvester ordering (harness/proto_fp8.py:61-64), scale 0.088388347648 = 1/sqrt(128)
 *     (kernel/exl3_grouped_prefill.cu:43), pre-scale by the per-expert sign vector
 *     (kernel/exl3_grouped_prefill.cu:113-114), epilogue H128 * scale * svh
 *     (kernel/exl3_grouped_prefill.cu:46-58, kernel/test_fat_v2.py:87-95).
 *   - SwiGLU clamp: g' = min(g, L), u' = clamp(u, -L, L), a = g'/(1+exp(-g')) * u'
 *     (kernel/exl3_grouped_prefill.cu:133-136).
 *   - Block table: kernel/exl3_grouped_prefill.cu:63-96 (build_blocks_kernel).
 *   - Stable expert sort: kernel/exl3_grouped_runtime.py:59-67.
 *
 * Trellis codebook — PARITY UNPINNED.  The reference decodes with exllamav3's dq_dispatch<4,1>
 * (K4 MCG codebook, commit c5d9c657), which is not vendored in the reference and not installed here.
 * This oracle (and the CUDA kernels) use the published QTIP "3INST" computed code instead
 * (Tseng et al. 2024, arXiv 2406.11235, "computed codes"): a 16-bit trellis state s is mapped to
 * x = (89226354*s + 64248484) mod 2^32, m = (x & 0x8fff8fff) ^ 0x3b603b60, and the weight is the
 * fp16 sum of m's two fp16 halves.  Tile format (this library's own; the CUDA decode uses the same):
 *   - one 16x16 tile = 64 int16 words = 32 little-endian u32 units = a 1024-bit cyclic stream;
 *     stream bit p is bit (31 - p%32) of unit p/32 (MSB first);
 *   - weight j (0..255) has state = stream bits [4j, 4j+16) (mod 1024), i.e. a tail-biting
 *     bitshift trellis with K=4 bits per weight and L=16 state bits;
 *   - weight j sits at (k = j % 16, n = j / 16) of the tile; tile (tk, tn) of a packed tensor
 *     [tiles_k, tiles_n, 64] covers W'[16tk:16tk+16, 16tn:16tn+16].
 * Everything downstream of the decode is pinned against the reference's own code (see
 * tests/golden/make_golden.py).
 *
 * Build: gcc -O2 -fPIC -shared -fopenmp (no -ffast-math: the Hadamard butterflies must round like IEEE
 * fp32).  Only the trellis decode of whole matrices runs on several threads.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>

#define ORC_HAD_SCALE 0.088388347648f

/* ------------------------------------------------------------------------------------ fp16 */
/* IEEE 754 binary16, round to nearest even. */
uint16_t orc_f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);           /* >= 65520 -> inf */
    if (ax < 0x38800000u)                                                 /* below 2^-14: subnormal */
    {
        if (ax < 0x33000000u) return (uint16_t) sign;                     /* below 2^-25 -> 0 */
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;                                  /* 14..24 */
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = (ax >> 13) - (112u << 10);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

float orc_h2f(uint16_t h)
{
    const uint32_t sign = ((uint32_t) h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0)
    {
        if (m == 0) x = sign;
        else
        {
            float f = (float) m * 5.9604644775390625e-08f;                /* m * 2^-24, exact */
            memcpy(&x, &f, 4);
            x |= sign;
        }
    }
    else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void orc_f2h_array(const float* src, uint16_t* dst, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) dst[i] = orc_f2h(src[i]);
}

void orc_h2f_array(const uint16_t* src, float* dst, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) dst[i] = orc_h2f(src[i]);
}

/* bf16 -> fp32 is exact; used for route weights given as bf16. */
static float bf2f(uint16_t b)
{
    uint32_t x = (uint32_t) b << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------------------ trellis */
static inline uint32_t unit32(const uint16_t* w, int u)
{
    return (uint32_t) w[2 * u] | ((uint32_t) w[2 * u + 1] << 16);
}

/* Literal definition: assemble the 16 state bits one at a time. */
uint32_t orc_trellis_state_bitwise(const uint16_t* tile_words, int j)
{
    uint32_t s = 0;
    for (int i = 0; i < 16; ++i)
    {
        const int p = (4 * j + i) & 1023;
        const uint32_t bit = (unit32(tile_words, p >> 5) >> (31 - (p & 31))) & 1u;
        s = (s << 1) | bit;
    }
    return s;
}

/* Same state from a 64-bit window of two consecutive units. */
uint32_t orc_trellis_state(const uint16_t* tile_words, int j)
{
    const int p0 = 4 * j;
    const int u = p0 >> 5, off = p0 & 31;
    const uint64_t window = ((uint64_t) unit32(tile_words, u) << 32) | unit32(tile_words, (u + 1) & 31);
    return (uint32_t)((window >> (48 - off)) & 0xffffu);
}

/* QTIP 3INST computed code: 16-bit state -> fp16 weight (bits). */
uint16_t orc_codebook(uint32_t state)
{
    const uint32_t x = state * 89226354u + 64248484u;
    const uint32_t m = (x & 0x8fff8fffu) ^ 0x3b603b60u;
    return orc_f2h(orc_h2f((uint16_t)(m & 0xffffu)) + orc_h2f((uint16_t)(m >> 16)));
}

/* One tile -> 256 fp16 weights in tile order j (k = j % 16, n = j / 16). */
void orc_decode_tile(const uint16_t* tile_words, uint16_t* out256)
{
    for (int j = 0; j < 256; ++j) out256[j] = orc_codebook(orc_trellis_state(tile_words, j));
}

/* packed [tiles_k, tiles_n, 64] int16 -> W' [K, N] fp16 (row-major, K = 16*tiles_k, N = 16*tiles_n).
 * Tiles decode independently, so the rows of tiles are split over OpenMP threads (same result for any
 * thread count). */
void orc_reconstruct(const uint16_t* packed, int tiles_k, int tiles_n, uint16_t* w)
{
    const int64_t N = 16 * (int64_t) tiles_n;
    #pragma omp parallel for schedule(static)
    for (int tk = 0; tk < tiles_k; ++tk)
    {
        uint16_t tile[256];
        for (int tn = 0; tn < tiles_n; ++tn)
        {
            orc_decode_tile(packed + ((int64_t) tk * tiles_n + tn) * 64, tile);
            for (int j = 0; j < 256; ++j)
                w[(int64_t)(16 * tk + (j & 15)) * N + 16 * tn + (j >> 4)] = tile[j];
        }
    }
}

/* Same, fp32 output (the CPU baseline multiplies in fp32). */
void orc_reconstruct_f32(const uint16_t* packed, int tiles_k, int tiles_n, float* w)
{
    const int64_t N = 16 * (int64_t) tiles_n;
    #pragma omp parallel for schedule(static)
    for (int tk = 0; tk < tiles_k; ++tk)
    {
        uint16_t tile[256];
        for (int tn = 0; tn < tiles_n; ++tn)
        {
            orc_decode_tile(packed + ((int64_t) tk * tiles_n + tn) * 64, tile);
            for (int j = 0; j < 256; ++j)
                w[(int64_t)(16 * tk + (j & 15)) * N + 16 * tn + (j >> 4)] = orc_h2f(tile[j]);
        }
    }
}

/* ------------------------------------------------------------------------------------ H128 */
/* Unnormalised Sylvester transform in place, radix-2 stages h = 1, 2, ..., 64 in that order; at each
 * stage the lower element of a pair becomes a+b and the upper a-b.  The GPU kernels apply the same
 * stages in the same order, so the fp32 results agree bit for bit. */
void orc_had128(float* v)
{
    for (int h = 1; h < 128; h <<= 1)
        for (int i = 0; i < 128; ++i)
            if (!(i & h))
            {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
}

/* Epilogue of the trellis GEMM on an fp32 [M, N] block (row stride ld): per row and per 128 columns,
 * v = H128(v) * 0.088388347648 * svh[col]  (kernel/exl3_grouped_prefill.cu:46-58). In place. */
void orc_had_epilogue(float* y, int64_t M, int N, int64_t ld, const uint16_t* svh)
{
    for (int64_t r = 0; r < M; ++r)
        for (int c0 = 0; c0 < N; c0 += 128)
        {
            float* v = y + r * ld + c0;
            orc_had128(v);
            for (int i = 0; i < 128; ++i)
            {
                float t = v[i] * ORC_HAD_SCALE;
                v[i] = t * orc_h2f(svh[c0 + i]);
            }
        }
}

/* row_had: dst[r, :] = fp16( H128( src[token_sorted[r] or r] (.) suh[expert_of_row[r]] ) * scale ),
 * per 128-column block (kernel/exl3_grouped_prefill.cu:101-115). */
void orc_row_had(const uint16_t* src, uint16_t* dst, int64_t rows, int K, const int64_t* token_sorted,
                 const int32_t* expert_of_row, const uint16_t* suh, int64_t suh_stride, int gather)
{
    float v[128];
    for (int64_t r = 0; r < rows; ++r)
    {
        const int64_t srow = gather ? token_sorted[r] : r;
        const uint16_t* s = suh + (int64_t) expert_of_row[r] * suh_stride;
        for (int b = 0; b < K; b += 128)
        {
            for (int i = 0; i < 128; ++i) v[i] = orc_h2f(src[srow * K + b + i]) * orc_h2f(s[b + i]);
            orc_had128(v);
            for (int i = 0; i < 128; ++i) dst[r * K + b + i] = orc_f2h(v[i] * ORC_HAD_SCALE);
        }
    }
}

/* Clamped SwiGLU of one element (kernel/exl3_grouped_prefill.cu:133-135). */
float orc_swiglu(float g, float u, float limit)
{
    const float gv = fminf(g, limit);
    const float uv = fminf(fmaxf(u, -limit), limit);
    return gv / (1.0f + expf(-gv)) * uv;
}

/* act_had: gu fp16 [rows, 2I] -> act fp16 [rows, I] (kernel/exl3_grouped_prefill.cu:118-141). */
void orc_act_had(const uint16_t* gu, uint16_t* act, int64_t rows, int I, const int32_t* expert_of_row,
                 const uint16_t* suh, int64_t suh_stride, float limit)
{
    float v[128];
    for (int64_t r = 0; r < rows; ++r)
    {
        const uint16_t* s = suh + (int64_t) expert_of_row[r] * suh_stride;
        const uint16_t* g = gu + r * 2 * (int64_t) I;
        const uint16_t* u = g + I;
        for (int b = 0; b < I; b += 128)
        {
            for (int i = 0; i < 128; ++i)
            {
                const uint16_t a = orc_f2h(orc_swiglu(orc_h2f(g[b + i]), orc_h2f(u[b + i]), limit));
                v[i] = orc_h2f(a) * orc_h2f(s[b + i]);
            }
            orc_had128(v);
            for (int i = 0; i < 128; ++i) act[r * I + b + i] = orc_f2h(v[i] * ORC_HAD_SCALE);
        }
    }
}

/* ------------------------------------------------------------------------------------ routing */
/* build_blocks (kernel/exl3_grouped_prefill.cu:63-96): per expert ceil(count/128) blocks in expert
 * order; block_expert[b] = e, block_row0[b] = row0[e] + 128*i; entries past the end get
 * block_expert = -1 and block_row0 untouched; meta = {n_blocks, n_rows}. */
void orc_build_blocks(const int32_t* counts, int n_experts, int max_blocks, int32_t* block_expert,
                      int32_t* block_row0, int32_t* meta)
{
    int row = 0, blk = 0;
    for (int e = 0; e < n_experts; ++e)
    {
        const int nblk = (counts[e] + 127) / 128;
        for (int i = 0; i < nblk; ++i)
        {
            const int b = blk + i;
            if (b < max_blocks)
            {
                block_expert[b] = e;
                block_row0[b] = row + i * 128;
            }
        }
        row += counts[e];
        blk += nblk;
    }
    meta[0] = blk;
    meta[1] = row;
    for (int b = blk; b < max_blocks; ++b) block_expert[b] = -1;
}

/* Stable sort of the flattened routing by expert (kernel/exl3_grouped_runtime.py:59-67):
 * order = argsort(ids.reshape(-1), stable=True); token_sorted = (order // topk) as int64;
 * weight_sorted = fp16(weights.reshape(-1)[order]); expert_of_row = ids[order] as int32;
 * counts = bincount; expert_row0 = exclusive cumsum.  weight_dtype: 0 fp32, 1 fp16, 2 bf16.
 * Ids outside [0, E) are not routed; their number is returned. */
int64_t orc_route_sort(const int64_t* ids, const void* weights, int weight_dtype, int64_t T, int topk,
                       int n_experts, int64_t* token_sorted, uint16_t* weight_sorted,
                       int32_t* expert_of_row, int32_t* counts, int32_t* expert_row0)
{
    const int64_t R = T * topk;
    int64_t invalid = 0;
    for (int e = 0; e < n_experts; ++e) counts[e] = 0;
    for (int64_t i = 0; i < R; ++i)
    {
        if (ids[i] < 0 || ids[i] >= n_experts) { invalid++; continue; }
        counts[ids[i]]++;
    }
    int32_t row = 0;
    int32_t* fill = (int32_t*) malloc(sizeof(int32_t) * (size_t)(n_experts > 0 ? n_experts : 1));
    for (int e = 0; e < n_experts; ++e) { expert_row0[e] = row; fill[e] = row; row += counts[e]; }
    for (int64_t i = 0; i < R; ++i)
    {
        const int64_t e = ids[i];
        if (e < 0 || e >= n_experts) continue;
        const int32_t pos = fill[e]++;
        token_sorted[pos] = i / topk;
        expert_of_row[pos] = (int32_t) e;
        float w;
        if (weight_dtype == 0) w = ((const float*) weights)[i];
        else if (weight_dtype == 1) w = orc_h2f(((const uint16_t*) weights)[i]);
        else w = bf2f(((const uint16_t*) weights)[i]);
        weight_sorted[pos] = orc_f2h(w);
    }
    free(fill);
    return invalid;
}
