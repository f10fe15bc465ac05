// attn_decode.cuh — split-KV GQA decode attention, one thread-block cluster
// per KV head (sm_100a).
//
// Replaces the upstream attention block of src/models/model.c:1226-1438:
// per query head, scores = (q . k_j) * (1/sqrt(hd)) (q_matmul_f32_avx2 +
// the scale at model.c:1376), causal mask -1e9 (q_causal_mask_f32_avx2),
// softmax (src/ops/avx2/softmax.c:17-132) and P.V — here over cache
// positions 0..valid-1 as the graph intends.  The softmax keeps upstream's
// numerics: the global row max first, then the polynomial exp on elements
// i < 8*floor(N/8) and expf on the tail (all expf when N < 8), where N is
// the row length of the upstream call (pos + seq_len); masked positions
// contribute exactly 0 upstream and are skipped here.  That exp is clamped,
// hence not multiplicative, so the row max is global before any exponential
// (no online-softmax rescaling).
//
// Cache layout (upstream get_kv_cache_ptr, model.c:700-740):
// [layer][kv_head][max_seq][K(hd) | V(hd)] fp32.
//
// Grid (CS, n_kv_heads), cluster (CS, 1, 1): the CS CTAs of a cluster share
// one KV head and split its valid positions into CS contiguous chunks; the
// G query heads of that KV head ride along, so every K/V row is read once.
// In each CTA a producer warp streams the chunk's K rows and then its V rows
// through a shared-memory ring — one tiled TMA copy per stage through a
// tensor map over the whole cache (box = SP rows x hd floats at the cache's
// row stride; this GPU's own memory, no multicast) — while 8 consumer warps
//   1. compute scores into shared memory and the chunk max, and store that
//      max into every CTA's shared memory (distributed shared memory),
//   | cluster barrier: each CTA takes the max of the CS maxima it holds
//   | (same values, same order everywhere, so the same global max),
//   2. turn scores into exponentials (upstream's index rule), sum them, and
//      accumulate partial P.V from the V rows (already streaming in); store
//      the sums into every CTA and each 1/CS slice of the partial outputs
//      into the CTA that finishes that slice,
//   | cluster barrier,
//   3. finish the slice from local shared memory: sum the CS partials (CTA
//      order) and multiply by 1/L.
// No CTA touches another's shared memory after the second barrier, so CTAs
// may leave as soon as they are done.
// Rows older than the current position do not depend on the previous kernel
// and are copied before the programmatic-dependency wait; the current row
// (written by the QKV epilogue just before) is copied after it.
#pragma once

#include <cuda.h>  // CUtensorMap

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

static constexpr int ATT_CWARPS = 8;                           // consumer warps
static constexpr int ATT_THREADS = ATT_CWARPS * 32 + 32;       // + producer warp
static constexpr int ATT_MAXG = 8;                             // query heads per KV head
static constexpr uint32_t ATT_STAGE_BYTES = 16384;             // one ring slot
static constexpr uint32_t ATT_MAX_SLOTS = 8;

struct AttnArgs {
    const float* q;          // [n_heads][hd] rotated queries
    uint32_t layer;          // cache plane z = layer * n_kv_heads + kv head
    float* out;              // [n_heads][hd]
    const StepParams* step;
    uint32_t n_heads, n_kv_heads, max_seq;
    uint32_t chunk_alloc;    // >= the longest chunk (whole stages of 16 KB / (4 hd) rows): scores per query head
    uint32_t slots;          // ring depth (2..ATT_MAX_SLOTS)
    float scale;             // 1/sqrtf(hd), computed on the host like upstream
    unsigned long long* trace;  // step-trace slot (null: off)
    // batched decode (grid z = sequence b): q, out and step advance by these
    // per sequence, and sequence b's cache planes follow the first b caches
    uint32_t seq_stride;     // floats of q / out per sequence
    uint32_t n_layers;       // planes per sequence = n_layers * n_kv_heads
    // paged caches (batched decode): sequence b's rows [r * page_rows, (r + 1) * page_rows)
    // live in page pages[b * pages_per_seq + r]; plane (page * n_layers + layer) * n_kv_heads + head
    const uint32_t* pages;   // null: contiguous caches
    uint32_t page_rows, pages_per_seq;
};

// ring[slots][16 KB] | sc[G][chunk_alloc] | ored[PG][G][hd]
__host__ __device__ inline size_t attn_smem_bytes(uint32_t G, uint32_t hd, uint32_t chunk_alloc,
                                                  uint32_t slots) {
    const uint32_t PG = (ATT_CWARPS * 32) / (hd / 4);
    return (size_t)slots * ATT_STAGE_BYTES + (size_t)G * chunk_alloc * 4 + (size_t)PG * G * hd * 4;
}

// Whole-warp calls only (.aligned): each reconverges its warp first.
__device__ __forceinline__ void cluster_arrive() {
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    __syncwarp();
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tiled TMA load of box (x, y, z) of a 3-D tensor map into shared memory,
// completing on `bar`.  x * 4 bytes is a multiple of 16 (x = 0 or hd).
__device__ __forceinline__ void tma_load_3d(void* dst_smem, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst_smem)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Store into CTA `rank`'s shared memory, at the address `p` has in ours.
__device__ __forceinline__ void st_dsmem(float* p, uint32_t rank, float v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
__device__ __forceinline__ void st_dsmem4(float* p, uint32_t rank, float4 v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(ra), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}


template <int HD, int G>
__global__ void __launch_bounds__(ATT_THREADS, G <= 4 ? 2 : 1)
    attn_decode_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap kv_map) {
    constexpr int NW = ATT_CWARPS, T = NW * 32;
    constexpr uint32_t RB = HD * 4;                  // bytes of one K or V row
    constexpr uint32_t SP = ATT_STAGE_BYTES / RB;    // rows per stage
    constexpr int LPP = HD / 16;                     // phase 1: lanes per row, 4 float4 each
    constexpr int PPW = 32 / LPP;                    // phase 1: rows per warp
    static_assert(SP == NW * PPW, "one phase-1 round per stage");
    constexpr int VQ = HD / 4;                       // phase 2: float4 columns of a V row
    constexpr int PG = T / VQ;                       // phase 2: row groups
    constexpr int PPG = SP / PG;                     // phase 2: rows per group per stage
    static_assert(PPG * PG == SP, "phase-2 split");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[ATT_MAX_SLOTS], empty[ATT_MAX_SLOTS];
    __shared__ float wred[NW][ATT_MAXG];
    __shared__ float gmx[ATT_MAXG], linv[ATT_MAXG];
    // filled by the other CTAs of the cluster (pushed before each cluster barrier)
    __shared__ float cmx[16][ATT_MAXG];                    // chunk maxima, by source CTA
    __shared__ float lgath[16][ATT_MAXG];                  // exponential sums, by source CTA
    __shared__ __align__(16) float pgath[ATT_MAXG * 128 + 16];  // [CS][per] partial outputs of my slice

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t CS = gridDim.x, r = blockIdx.x, h = blockIdx.y;  // cluster = one grid row
    const uint32_t CA = a.chunk_alloc, SL = a.slots;
    uint8_t* ring = smem;
    float* sc = reinterpret_cast<float*>(smem + (size_t)SL * ATT_STAGE_BYTES);  // [G][CA]
    float4* ored = reinterpret_cast<float4*>(sc + (size_t)G * CA);              // [PG][G][VQ]

    if (tid == 0) {
        trace_mark(a.trace, 0);
        for (uint32_t s = 0; s < SL; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    // Step scalars come from the previous graph replay or a host copy, both
    // complete before this grid starts.
    const uint32_t bz = blockIdx.z;  // sequence (batched decode; 0 otherwise)
    const StepParams* stp = a.step + bz;
    const uint32_t valid = stp->valid, N = stp->n_row, cur = stp->pos;
    // CTA r takes whole ring stages [n_st r / CS, n_st (r+1) / CS) of the
    // valid rows, so only the last stage of the sequence is a partial box
    const uint32_t n_st = (valid + SP - 1) / SP;
    const uint32_t p0 = min(n_st * r / CS * SP, valid), p1 = min(n_st * (r + 1) / CS * SP, valid);
    const int plane = (int)(((size_t)bz * a.n_layers + a.layer) * a.n_kv_heads + h);
    const float* qseq = a.q + (size_t)bz * a.seq_stride;
    float* oseq = a.out + (size_t)bz * a.seq_stride;

    if (warp == NW) {
        // ---- producer: K rows of the chunk, then its V rows ------------------
        cluster_arrive();  // barrier 1 does not wait for the producer's copies
        const uint64_t pol = l2_evict_first_policy();
        uint32_t s = 0, ph = 0, k = 0;
        bool waited = false, ok = true;
        for (uint32_t pass = 0; pass < 2 && ok; ++pass) {
            for (uint32_t sp0 = p0; sp0 < p1; sp0 += SP, ++k) {
                if (k >= SL && !mbar_wait(&empty[s], ph ^ 1, QDEV_WAIT_EMPTY_TIMEOUT)) {
                    ok = false;
                    break;
                }
                const uint32_t n = min(SP, p1 - sp0);
                if (!waited && sp0 + n > cur) {
                    pdl_wait();
                    waited = true;
                }
                // the whole box arrives (rows past the chunk, or past max_seq as
                // zeros, are loaded and ignored)
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], ATT_STAGE_BYTES);
                    // a stage never straddles pages (page_rows is a multiple of SP)
                    int y = (int)sp0, z = plane;
                    if (a.pages) {
                        const uint32_t pg = __ldg(a.pages + (size_t)bz * a.pages_per_seq + sp0 / a.page_rows);
                        y = (int)(sp0 % a.page_rows);
                        z = (int)(((size_t)pg * a.n_layers + a.layer) * a.n_kv_heads + h);
                    }
                    tma_load_3d(ring + (size_t)s * ATT_STAGE_BYTES, &kv_map, (int)(pass * HD), y, z, &full[s], pol);
                }
                __syncwarp();
                if (++s == SL) {
                    s = 0;
                    ph ^= 1;
                }
            }
        }
        if (!waited) pdl_wait();  // every thread waits: the grid ends after its predecessor
        cluster_wait();
        cluster_arrive();
        cluster_wait();
        return;
    }

    // ---- consumers -----------------------------------------------------------------
    pdl_wait();  // q is the previous kernel's output
    if (tid == 0) trace_mark(a.trace, 1);

    uint32_t s = 0, ph = 0;
    // phase 1: scores and chunk max
    {
        const uint32_t sub = lane % LPP, slot = lane / LPP, row = warp * PPW + slot;
        // lane `sub` of a row takes float4s sub, sub + LPP, ... of q and K, so
        // the 8 lanes of each shared-memory phase read 128 contiguous bytes;
        // its q float4s stay in registers for the whole chunk
        float4 qr[G][4];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                qr[g][i] = reinterpret_cast<const float4*>(qseq + (size_t)(h * G + g) * HD)[sub + i * LPP];
        float mx[G];
#pragma unroll
        for (int g = 0; g < G; ++g) mx[g] = -INFINITY;
        uint32_t kst = 0;
        for (uint32_t sp0 = p0; sp0 < p1; sp0 += SP) {
            mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
            ++kst;
            const uint32_t p = sp0 + row;
            const bool live = p < p1;
            const float4* kr = reinterpret_cast<const float4*>(ring + (size_t)s * ATT_STAGE_BYTES + row * RB) + sub;
            float4 k4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) k4[i] = kr[i * LPP];
            // all heads' chains interleaved (independent accumulators), then
            // the cross-lane sums level by level
            float d[G];
#pragma unroll
            for (int g = 0; g < G; ++g) d[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 qv = qr[g][i];
                    d[g] = __fmaf_rn(qv.x, k4[i].x, d[g]);
                    d[g] = __fmaf_rn(qv.y, k4[i].y, d[g]);
                    d[g] = __fmaf_rn(qv.z, k4[i].z, d[g]);
                    d[g] = __fmaf_rn(qv.w, k4[i].w, d[g]);
                }
            }
#pragma unroll
            for (int o = LPP / 2; o > 0; o >>= 1)
#pragma unroll
                for (int g = 0; g < G; ++g) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
            if (live) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float sv = __fmul_rn(d[g], a.scale);
                    if (sub == 0) sc[g * CA + (p - p0)] = sv;
                    mx[g] = fmaxf(mx[g], sv);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == SL) {
                s = 0;
                ph ^= 1;
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float m = warp_max(mx[g]);
            if (lane == 0) wred[warp][g] = m;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        // push this chunk's max of each query head to every CTA of the cluster
        for (uint32_t i = tid; i < CS * G; i += T) {
            const uint32_t g = i % G;
            float m = -INFINITY;
            for (int w = 0; w < NW; ++w) m = fmaxf(m, wred[w][g]);
            st_dsmem(&cmx[r][g], i / G, m);
        }
    }
    cluster_arrive();
    cluster_wait();

    // phase 2: global max, exponentials (upstream index rule), sums, partial P.V
    if (tid < G) {
        float m = -INFINITY;
        for (uint32_t rr = 0; rr < CS; ++rr) m = fmaxf(m, cmx[rr][tid]);
        gmx[tid] = m;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(T));
    const uint32_t len = p1 - p0;
    const uint32_t nvec = N < 8 ? 0u : (N / 8) * 8;
    for (uint32_t i = tid; i < G * len; i += T) {
        const uint32_t g = i / len, pp = i % len;
        const float x = __fsub_rn(sc[g * CA + pp], gmx[g]);
        sc[g * CA + pp] = (p0 + pp) < nvec ? exp_poly(x) : expf(x);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(T));
    if (warp < G) {
        float l = 0.0f;
        for (uint32_t pp = lane; pp < len; pp += 32) l += sc[warp * CA + pp];
        l = warp_sum(l);
        // push this chunk's sum to every CTA
        for (uint32_t rr = lane; rr < CS; rr += 32) st_dsmem(&lgath[r][warp], rr, l);
    }
    {
        const uint32_t dq = tid % VQ, pg = tid / VQ;
        float4 o[G];
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t vst = 12;
        for (uint32_t sp0 = p0; sp0 < p1; sp0 += SP) {
            mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
            ++vst;
            const uint8_t* stage = ring + (size_t)s * ATT_STAGE_BYTES;
#pragma unroll
            for (int j = 0; j < PPG; ++j) {
                const uint32_t i = pg * PPG + j, p = sp0 + i;
                if (p >= p1) break;
                const float4 v = reinterpret_cast<const float4*>(stage + i * RB)[dq];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float e = sc[g * CA + (p - p0)];
                    o[g].x = __fmaf_rn(e, v.x, o[g].x);
                    o[g].y = __fmaf_rn(e, v.y, o[g].y);
                    o[g].z = __fmaf_rn(e, v.z, o[g].z);
                    o[g].w = __fmaf_rn(e, v.w, o[g].w);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == SL) {
                s = 0;
                ph ^= 1;
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) ored[((size_t)pg * G + g) * VQ + dq] = o[g];
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        for (uint32_t i = tid; i < G * VQ; i += T) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < PG; ++q) {
                const float4 t = ored[(size_t)q * G * VQ + i];
                acc.x += t.x;
                acc.y += t.y;
                acc.z += t.z;
                acc.w += t.w;
            }
            // outputs 4i..4i+3 belong to CTA 4i / per (per is a multiple of 8)
            const uint32_t per = G * HD / CS, o = 4 * i;
            st_dsmem4(&pgath[r * per + o % per], o / per, acc);
        }
    }
    cluster_arrive();
    cluster_wait();

    // phase 3: this CTA's slice of the outputs, from the partials and sums
    // every CTA pushed here (summed in CTA order)
    {
        const uint32_t per = G * HD / CS, o0 = r * per;
        if (tid < G) {
            float l = 0.0f;
            for (uint32_t rr = 0; rr < CS; ++rr) l += lgath[rr][tid];
            linv[tid] = __fdiv_rn(1.0f, l);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        for (uint32_t k = tid; k < per; k += T) {
            float acc = 0.0f;
            for (uint32_t rr = 0; rr < CS; ++rr) acc += pgath[rr * per + k];
            oseq[(size_t)h * G * HD + o0 + k] = __fmul_rn(acc, linv[(o0 + k) / HD]);
        }
    }
    // (no shared memory of another CTA is touched after the second barrier)
    if (tid == 0) trace_mark(a.trace, 2);
}

}  // namespace qb200
