// attn_decode.cuh — split-KV decode attention over the HBM KV cache (sm_100a).
//
// Replaces the upstream attention block of src/models/model.c:1226-1438:
// per query head, scores = (q . k_j) * (1/sqrt(hd)) (q_matmul_f32_avx2 +
// the scale at model.c:1376), causal mask -1e9 (q_causal_mask_f32_avx2),
// softmax (src/ops/avx2/softmax.c:17-132) and P.V — here over cache
// positions 0..valid-1 as the graph intends.  The softmax keeps upstream's
// numerics: the global row max first, then the polynomial exp on elements
// i < 8*floor(N/8) and expf on the tail (all expf when N < 8), where N is
// the row length of the upstream call (pos + seq_len).  That exp is not
// multiplicative, so the row max is global before any exponential (no
// online-softmax rescaling).
//
// Cache layout (upstream get_kv_cache_ptr, model.c:700-740):
// [layer][kv_head][max_seq][K(hd) | V(hd)] fp32.
//
// One kernel, grid (n_kv_heads, NC), launched cooperatively so all CTAs are
// co-resident.  The G query heads of a KV head share its CTAs, so every K/V
// row is read once.  The valid positions are split over the first n_act <=
// NC CTAs of each head; a CTA issues all K and V loads of its chunk (in
// sub-chunks of 64 positions) before it needs them, keeps its scores in
// shared memory, and passes three phases:
//   1. scores (HD/16 lanes per position), chunk max -> global | head barrier
//   2. global max, exponentials, partial P.V and sums -> global | head barrier
//   3. each CTA combines a slice of the G*HD outputs.
// Barriers are atomic counters per head with bounded spins; the last CTA of
// a head resets that head's counters for the next launch.
#pragma once

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

static constexpr int ATT_THREADS = 256;
static constexpr int ATT_MAXG = 8;        // query heads per KV head supported
static constexpr int ATT_MIN_CHUNK = 32;  // positions per CTA before using more CTAs
static constexpr int ATT_SUB = 64;        // positions per register-resident sub-chunk

struct AttnArgs {
    const float* q;          // [n_heads][hd] rotated queries
    const float* kv_layer;   // this layer's cache base
    float* cmax;             // [n_heads][NC]
    float* opart;            // [n_heads][NC][hd]
    float* lpart;            // [n_heads][NC]
    uint32_t* sync;          // [n_kv_heads][4] counters, zero between launches
    float* out;              // [n_heads][hd]
    const StepParams* step;
    uint32_t n_heads, n_kv_heads, max_seq, n_chunks;  // n_chunks = NC (grid.y)
    uint32_t chunk_alloc;    // >= ceil(max_seq / NC): shared scores per head
    float scale;             // 1/sqrtf(hd), computed on the host like upstream
    unsigned long long* trace;  // step-trace slot (null: off)
};

__host__ __device__ inline size_t attn_smem_bytes(uint32_t G, uint32_t chunk_alloc) {
    return (size_t)G * chunk_alloc * 4;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// CTA-wide wait until *ctr >= target (bounded); thread 0 polls.
__device__ __forceinline__ void head_barrier(uint32_t* ctr, uint32_t target) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
        uint32_t i = 0;
        while (ld_acquire(ctr) < target) {
            if (++i > (1u << 24)) {
                qdev_fail(QDEV_COMBINE_TIMEOUT);
                break;
            }
            __nanosleep(20);
        }
    }
    __syncthreads();
}

#ifdef QB200_ATTN_PHASES  // experiment builds only: per-CTA phase timestamps
__device__ unsigned long long g_attn_phase[1024 * 8];
#define ATTN_PHASE(i)                                                                         \
    do {                                                                                      \
        if (threadIdx.x == 0) g_attn_phase[(blockIdx.y * gridDim.x + blockIdx.x) * 8 + (i)] = gtimer(); \
    } while (0)
#else
#define ATTN_PHASE(i) ((void)0)
#endif

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS, 2) attn_decode_kernel(const AttnArgs a) {
    constexpr int LPP = HD / 16;                 // lanes per K row (16 floats each)
    constexpr int PPW = 32 / LPP;                // positions per warp per K round
    constexpr int NW = ATT_THREADS / 32;
    constexpr int SUB = NW * PPW > ATT_SUB ? NW * PPW : ATT_SUB;  // positions per sub-chunk
    constexpr int KR = SUB / (NW * PPW);         // K rounds per sub-chunk
    constexpr int VL = HD / 4;                   // lanes per V row (float4 each)
    constexpr int PL = ATT_THREADS / VL;         // V rows in flight per round
    constexpr int VR = SUB / PL;                 // V rounds per sub-chunk
    static_assert(KR >= 1 && VR >= 1, "sub-chunk too small");
    extern __shared__ __align__(16) float sc[];  // [G][chunk_alloc]: scores, then e
    __shared__ __align__(16) float qs[ATT_MAXG][HD];
    __shared__ float wred[NW][ATT_MAXG];
    __shared__ float gmax[ATT_MAXG];
    __shared__ __align__(16) float4 ored[PL][ATT_MAXG][VL];
    __shared__ float lsum[ATT_MAXG];
    if (threadIdx.x == 0) trace_mark(a.trace, 0);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(a.trace, 1);
    ATTN_PHASE(0);
    const uint32_t h = blockIdx.x, c = blockIdx.y;
    const uint32_t G = a.n_heads / a.n_kv_heads;
    const uint32_t valid = a.step->valid, N = a.step->n_row;
    uint32_t n_act = (valid + ATT_MIN_CHUNK - 1) / ATT_MIN_CHUNK;
    n_act = n_act < a.n_chunks ? n_act : a.n_chunks;
    if (c >= n_act) return;
    const uint32_t chunk = (valid + n_act - 1) / n_act;
    const uint32_t p0 = c * chunk, p1 = min(p0 + chunk, valid);
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* slab = a.kv_layer + (size_t)h * a.max_seq * 2 * HD;
    uint32_t* ctr = a.sync + 4 * h;
    const uint32_t CA = a.chunk_alloc;

    // V of the first sub-chunk: in flight from the start, used in phase 2
    const uint32_t vl = tid % VL, pl = tid / VL;
    float4 vreg[VR];
#pragma unroll
    for (int r = 0; r < VR; ++r) {
        const uint32_t p = p0 + pl + r * PL;
        vreg[r] = p < p1 ? __ldg(reinterpret_cast<const float4*>(slab + (size_t)p * 2 * HD + HD) + vl)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (uint32_t i = tid; i < G * HD; i += ATT_THREADS)
        qs[i / HD][i % HD] = a.q[(size_t)(h * G) * HD + i];
    __syncthreads();
    ATTN_PHASE(1);

    // ---- phase 1: scores + chunk max ------------------------------------------
    {
        const uint32_t sub = lane % LPP, slot = lane / LPP;
        float mx[ATT_MAXG];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) mx[g] = -INFINITY;
        for (uint32_t sp0 = p0; sp0 < p1; sp0 += SUB) {
            const uint32_t sp1 = min(sp0 + SUB, p1);
            float4 k4[KR][4];
#pragma unroll
            for (int r = 0; r < KR; ++r) {
                const uint32_t p = sp0 + r * NW * PPW + warp * PPW + slot;
                const float4* kp = reinterpret_cast<const float4*>(slab + (size_t)(p < sp1 ? p : sp0) * 2 * HD + sub * 16);
#pragma unroll
                for (int i = 0; i < 4; ++i) k4[r][i] = __ldg(kp + i);
            }
#pragma unroll
            for (int r = 0; r < KR; ++r) {
                const uint32_t p = sp0 + r * NW * PPW + warp * PPW + slot;
                const bool live = p < sp1;
#pragma unroll
                for (int g = 0; g < ATT_MAXG; ++g) {
                    if (g >= (int)G) break;
                    const float4* q4 = reinterpret_cast<const float4*>(&qs[g][sub * 16]);
                    float d = 0.0f;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 qv = q4[i];
                        d = __fmaf_rn(qv.x, k4[r][i].x, d);
                        d = __fmaf_rn(qv.y, k4[r][i].y, d);
                        d = __fmaf_rn(qv.z, k4[r][i].z, d);
                        d = __fmaf_rn(qv.w, k4[r][i].w, d);
                    }
#pragma unroll
                    for (int o = LPP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    const float s = __fmul_rn(d, a.scale);
                    if (live) {
                        if (sub == 0) sc[g * CA + (p - p0)] = s;
                        mx[g] = fmaxf(mx[g], s);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) {
            if (g >= (int)G) break;
            const float m = warp_max(mx[g]);
            if (lane == 0) wred[warp][g] = m;
        }
        __syncthreads();
        if (tid < G) {
            float m = -INFINITY;
            for (int w = 0; w < NW; ++w) m = fmaxf(m, wred[w][tid]);
            a.cmax[(size_t)(h * G + tid) * a.n_chunks + c] = m;
        }
    }
    ATTN_PHASE(2);
    head_barrier(ctr + 0, n_act);
    ATTN_PHASE(3);

    // ---- phase 2: exponentials (upstream index rule) + partial P.V -------------
    if (warp < G) {
        float m = -INFINITY;
        for (uint32_t i = lane; i < n_act; i += 32)
            m = fmaxf(m, __ldcg(&a.cmax[(size_t)(h * G + warp) * a.n_chunks + i]));
        m = warp_max(m);
        if (lane == 0) gmax[warp] = m;
    }
    __syncthreads();
    const uint32_t len = p1 - p0;
    const uint32_t nvec = N < 8 ? 0u : (N / 8) * 8;
    for (uint32_t i = tid; i < G * len; i += ATT_THREADS) {
        const uint32_t g = i / len, pp = i % len;
        const float x = __fsub_rn(sc[g * CA + pp], gmax[g]);
        sc[g * CA + pp] = (p0 + pp) < nvec ? exp_poly(x) : expf(x);
    }
    __syncthreads();
    if (warp < G) {
        float l = 0.0f;
        for (uint32_t pp = lane; pp < len; pp += 32) l += sc[warp * CA + pp];
        l = warp_sum(l);
        if (lane == 0) lsum[warp] = l;
    }
    {
        float4 o[ATT_MAXG];
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g) o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t sp0 = p0; sp0 < p1; sp0 += SUB) {
            if (sp0 != p0) {  // later sub-chunks (long contexts): load now
#pragma unroll
                for (int r = 0; r < VR; ++r) {
                    const uint32_t p = sp0 + pl + r * PL;
                    vreg[r] = p < p1 ? __ldg(reinterpret_cast<const float4*>(slab + (size_t)p * 2 * HD + HD) + vl)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int r = 0; r < VR; ++r) {
                const uint32_t p = sp0 + pl + r * PL;
                if (p >= p1) break;
                const float4 v = vreg[r];
#pragma unroll
                for (int g = 0; g < ATT_MAXG; ++g) {
                    if (g >= (int)G) break;
                    const float e = sc[g * CA + (p - p0)];
                    o[g].x = __fmaf_rn(e, v.x, o[g].x);
                    o[g].y = __fmaf_rn(e, v.y, o[g].y);
                    o[g].z = __fmaf_rn(e, v.z, o[g].z);
                    o[g].w = __fmaf_rn(e, v.w, o[g].w);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < ATT_MAXG; ++g)
            if (g < (int)G) ored[pl][g][vl] = o[g];
        __syncthreads();
        for (uint32_t i = tid; i < G * VL; i += ATT_THREADS) {
            const uint32_t g = i / VL, j = i % VL;
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < PL; ++q) {
                const float4 t = ored[q][g][j];
                s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
            }
            reinterpret_cast<float4*>(a.opart + ((size_t)(h * G + g) * a.n_chunks + c) * HD)[j] = s;
        }
        if (tid < G) a.lpart[(size_t)(h * G + tid) * a.n_chunks + c] = lsum[tid];
    }
    ATTN_PHASE(4);
    head_barrier(ctr + 1, n_act);
    ATTN_PHASE(5);

    // ---- phase 3: this CTA's slice of the outputs --------------------------------
    // The partials sit in L2; chunk sums are spread over lanes so every load
    // of a warp is in flight at once.
    {
        if (warp < G) {  // softmax denominators
            float l = 0.0f;
            for (uint32_t k = lane; k < n_act; k += 32)
                l += __ldcg(&a.lpart[(size_t)(h * G + warp) * a.n_chunks + k]);
            l = warp_sum(l);
            if (lane == 0) gmax[warp] = __fdiv_rn(1.0f, l);  // gmax now holds 1/L
        }
        __syncthreads();
        const uint32_t total = G * HD;
        const uint32_t per = (total + n_act - 1) / n_act;
        const uint32_t o0 = c * per, o1 = min(o0 + per, total);
        if (n_act <= 8) {
            for (uint32_t i = o0 + tid; i < o1; i += ATT_THREADS) {
                const uint32_t g = i / HD, d = i % HD;
                const size_t row = (size_t)(h * G + g) * a.n_chunks;
                float s = 0.0f;
#pragma unroll 8
                for (uint32_t k = 0; k < n_act; ++k) s += __ldcg(&a.opart[(row + k) * HD + d]);
                a.out[(size_t)(h * G + g) * HD + d] = __fmul_rn(s, gmax[g]);
            }
        } else {
            for (uint32_t i = o0 + warp; i < o1; i += NW) {
                const uint32_t g = i / HD, d = i % HD;
                const size_t row = (size_t)(h * G + g) * a.n_chunks;
                float s = 0.0f;
                for (uint32_t k = lane; k < n_act; k += 32) s += __ldcg(&a.opart[(row + k) * HD + d]);
                s = warp_sum(s);
                if (lane == 0) a.out[(size_t)(h * G + g) * HD + d] = __fmul_rn(s, gmax[g]);
            }
        }
    }
    // last CTA of the head resets the counters for the next launch
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(ctr + 2, 1u) == n_act - 1) {
            ctr[0] = 0u;
            ctr[1] = 0u;
            ctr[2] = 0u;
            __threadfence();
        }
        trace_mark(a.trace, 2);
    }
    ATTN_PHASE(6);
}

}  // namespace qb200
