// attn_decode.cuh — split-KV decode attention over the HBM KV cache (sm_100a).
//
// Replaces the upstream attention block of src/models/model.c:1226-1438:
// per query head, scores = (q . k_j) * (1/sqrt(hd)) (q_matmul_f32_avx2 +
// the scale at model.c:1376), causal mask -1e9 (q_causal_mask_f32_avx2),
// softmax (src/ops/avx2/softmax.c:17-132) and P.V — here over cache
// positions 0..valid-1 as the graph intends.  The softmax keeps upstream's
// numerics: the global row max first, then the polynomial exp on elements
// i < 8*floor(N/8) and expf on the tail (all expf when N < 8), where N is
// the row length of the upstream call (pos + seq_len).  Because that exp is
// not multiplicative, the max is taken over the whole row before any
// exponential (two kernels, not an online softmax).
//
// Cache layout (upstream get_kv_cache_ptr, model.c:700-740):
// [layer][kv_head][max_seq][K(hd) | V(hd)] fp32.
//
// attn_scores: grid (n_kv_heads, n_chunks of ATT_CH positions); the G query
//   heads sharing a KV head are packed in one CTA, each K row is read once.
//   HD/16 lanes cooperate on one position (16 elements each).
// attn_pv: same grid; exponentials of the chunk, partial P.V and partial
//   sums, then the last CTA of each KV head (atomic ticket) combines the
//   chunks and resets its ticket for the next call.
#pragma once

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

static constexpr int ATT_CH = 64;     // positions per chunk
static constexpr int ATT_THREADS = 128;
static constexpr int ATT_MAXG = 8;    // query heads per KV head supported

struct AttnArgs {
    const float* q;          // [n_heads][hd] rotated queries
    const float* kv_layer;   // this layer's cache base
    float* scores;           // [n_heads][max_seq]
    float* cmax;             // [n_heads][n_chunks]
    float* opart;            // [n_heads][n_chunks][hd]
    float* lpart;            // [n_heads][n_chunks]
    uint32_t* ticket;        // [n_kv_heads], zero between calls
    float* out;              // [n_heads][hd]
    const StepParams* step;
    uint32_t n_heads, n_kv_heads, max_seq, n_chunks;
    float scale;             // 1/sqrtf(hd), computed on the host like upstream
};

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_scores_kernel(const AttnArgs a) {
    constexpr int LPP = HD / 16;          // lanes per position
    constexpr int PPW = 32 / LPP;         // positions per warp step
    __shared__ __align__(16) float qs[ATT_MAXG][HD];
    __shared__ float wmax[ATT_THREADS / 32][ATT_MAXG];
    pdl_trigger();
    pdl_wait();
    const uint32_t h = blockIdx.x, chunk = blockIdx.y;
    const uint32_t G = a.n_heads / a.n_kv_heads;
    const uint32_t valid = a.step->valid;
    const uint32_t p0 = chunk * ATT_CH;
    if (p0 >= valid) return;
    const uint32_t p1 = min(p0 + ATT_CH, valid);
    for (uint32_t i = threadIdx.x; i < G * HD; i += ATT_THREADS)
        qs[i / HD][i % HD] = a.q[(size_t)(h * G) * HD + i];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t sub = lane % LPP, slot = lane / LPP;
    float mx[ATT_MAXG];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) mx[g] = -INFINITY;
    const float* base = a.kv_layer + (size_t)h * a.max_seq * 2 * HD + sub * 16;
    for (uint32_t p = p0 + warp * PPW + slot; p - slot < p1; p += (ATT_THREADS / 32) * PPW) {
        const bool live = p < p1;
        float4 k4[4];
        const float4* kp = reinterpret_cast<const float4*>(base + (size_t)(live ? p : p0) * 2 * HD);
#pragma unroll
        for (int i = 0; i < 4; ++i) k4[i] = kp[i];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) {
            if (g >= (int)G) break;
            const float4* q4 = reinterpret_cast<const float4*>(&qs[g][sub * 16]);
            float d = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 qv = q4[i];
                d = __fmaf_rn(qv.x, k4[i].x, d);
                d = __fmaf_rn(qv.y, k4[i].y, d);
                d = __fmaf_rn(qv.z, k4[i].z, d);
                d = __fmaf_rn(qv.w, k4[i].w, d);
            }
#pragma unroll
            for (int o = LPP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            const float s = __fmul_rn(d, a.scale);
            if (live) {
                if (sub == 0) a.scores[(size_t)(h * G + g) * a.max_seq + p] = s;
                mx[g] = fmaxf(mx[g], s);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) {
        if (g >= (int)G) break;
        float m = warp_max(mx[g]);
        if (lane == 0) wmax[warp][g] = m;
    }
    __syncthreads();
    if (threadIdx.x < G) {
        float m = -INFINITY;
        for (int w = 0; w < ATT_THREADS / 32; ++w) m = fmaxf(m, wmax[w][threadIdx.x]);
        a.cmax[(size_t)(h * G + threadIdx.x) * a.n_chunks + chunk] = m;
    }
}

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_pv_kernel(const AttnArgs a) {
    constexpr int PS = ATT_THREADS / HD;  // position lanes
    __shared__ float e[ATT_MAXG][ATT_CH];
    __shared__ float gmax[ATT_MAXG];
    __shared__ float red[PS][ATT_MAXG][HD];
    __shared__ uint32_t last;
    pdl_trigger();
    pdl_wait();
    const uint32_t h = blockIdx.x, chunk = blockIdx.y;
    const uint32_t G = a.n_heads / a.n_kv_heads;
    const uint32_t valid = a.step->valid, N = a.step->n_row;
    const uint32_t n_act = (valid + ATT_CH - 1) / ATT_CH;
    const uint32_t p0 = chunk * ATT_CH;
    if (p0 >= valid) return;
    const uint32_t p1 = min(p0 + ATT_CH, valid);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // global row max per head from the chunk maxima
    for (uint32_t g = warp; g < G; g += ATT_THREADS / 32) {
        float m = -INFINITY;
        for (uint32_t c = lane; c < n_act; c += 32)
            m = fmaxf(m, a.cmax[(size_t)(h * G + g) * a.n_chunks + c]);
        m = warp_max(m);
        if (lane == 0) gmax[g] = m;
    }
    __syncthreads();
    // exponentials with upstream's index rule
    const uint32_t nvec = N < 8 ? 0u : (N / 8) * 8;
    for (uint32_t i = threadIdx.x; i < G * ATT_CH; i += ATT_THREADS) {
        const uint32_t g = i / ATT_CH, p = p0 + i % ATT_CH;
        float v = 0.0f;
        if (p < p1) {
            const float x = __fsub_rn(a.scores[(size_t)(h * G + g) * a.max_seq + p], gmax[g]);
            v = p < nvec ? exp_poly(x) : expf(x);
        }
        e[g][i % ATT_CH] = v;
    }
    __syncthreads();
    static_assert(ATT_CH == 64, "partial sums assume two elements per lane");
    for (uint32_t g = warp; g < G; g += ATT_THREADS / 32) {  // partial softmax sums
        float s = e[g][lane] + e[g][lane + 32];
        s = warp_sum(s);
        if (lane == 0) a.lpart[(size_t)(h * G + g) * a.n_chunks + chunk] = s;
    }
    // partial P.V
    const uint32_t d = threadIdx.x % HD, ps = threadIdx.x / HD;
    float o[ATT_MAXG];
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g) o[g] = 0.0f;
    const float* vb = a.kv_layer + (size_t)h * a.max_seq * 2 * HD + HD + d;
    for (uint32_t p = p0 + ps; p < p1; p += PS) {
        const float v = vb[(size_t)p * 2 * HD];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g)
            if (g < (int)G) o[g] = __fmaf_rn(e[g][p - p0], v, o[g]);
    }
#pragma unroll
    for (int g = 0; g < ATT_MAXG; ++g)
        if (g < (int)G) red[ps][g][d] = o[g];
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < G * HD; i += ATT_THREADS) {
        const uint32_t g = i / HD, dd = i % HD;
        float s = 0.0f;
        for (int q = 0; q < PS; ++q) s += red[q][g][dd];
        a.opart[((size_t)(h * G + g) * a.n_chunks + chunk) * HD + dd] = s;
    }
    // last CTA of this KV head combines the chunks
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = (atomicAdd(&a.ticket[h], 1u) == n_act - 1) ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (uint32_t i = threadIdx.x; i < G * HD; i += ATT_THREADS) {
        const uint32_t g = i / HD, dd = i % HD;
        const size_t row = (size_t)(h * G + g) * a.n_chunks;
        float l = 0.0f, s = 0.0f;
        for (uint32_t c = 0; c < n_act; ++c) {
            l += __ldcg(&a.lpart[row + c]);
            s += __ldcg(&a.opart[(row + c) * HD + dd]);
        }
        a.out[(size_t)(h * G + g) * HD + dd] = __fmul_rn(s, __fdiv_rn(1.0f, l));
    }
    if (threadIdx.x == 0) a.ticket[h] = 0u;
}

}  // namespace qb200
