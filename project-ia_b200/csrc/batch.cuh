// batch.cuh — batched decode: B <= 16 sequences advance one token per step,
// every weight streamed from HBM once for all of them.
//
// Upstream decodes one sequence per llama_forward call (include/qorus.h:
// 212-219, src/main.c:994-1131); the same per-token graph (model.c:
// 1655-1850) runs here for B sequences at once.  Each sequence keeps its own
// KV cache in upstream's layout; the caches sit back to back.
//
// Q4_0 GEMV with B input columns (q4_batch_kernel).  The weights stay in the
// decode slab tiles (gemv_q4.cuh).  Per 32-row x 32-column tile a warp runs
// mma.sync m16n8k16 (f16 in, f32 accumulate) with
//   A = the nibbles minus 8 as fp16 — exact integers, converted with a byte
//       permute that places each nibble under the fp16 exponent of 1024 and
//       one packed subtract of 1032;
//   B = the inputs as fp16 halves hi + lo (v = hi + lo to 22 bits) after a
//       power-of-two scale per input row (batch_xprep_kernel);
// so every product is exact and the block's sum is an fp32 sum of 64 terms;
// the block is then scaled by the weight scale in fp32 registers — the same
// arithmetic as an fp32 dot product in another summation order.  The K order
// inside a block is permuted identically in A and B so that a lane's 16
// tile bytes feed its A fragments directly.  A CTA owns a range of whole
// slabs and streams up to 4 of them at a time block-major, so each block's
// input fragments (2 KB for 16 inputs, read from L2) serve all 4 slabs.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

static constexpr uint32_t BT_MAXB = 16;    // sequences per batch
static constexpr int BT_WARPS = 8;         // consumer warps (12 and 16 measured no faster)
static constexpr int BT_THREADS = BT_WARPS * 32 + 32;
static constexpr uint32_t BT_NS = 4;       // slabs streamed together
static constexpr uint32_t BT_SB = 16;      // blocks per ring stage
static constexpr uint32_t BT_STAGES = 3;
static constexpr uint32_t BT_STAGE_BYTES = BT_NS * BT_SB * GEMV_BLOCK_BYTES;  // 40 KB
static constexpr size_t BT_RED_BYTES = (size_t)BT_WARPS * BT_NS * 32 * BT_MAXB * 4;  // 64 KB
static constexpr size_t BT_SMEM = (size_t)BT_STAGES * BT_STAGE_BYTES + BT_RED_BYTES + 256;
// input fragments: per (32-block, group of 8 inputs, lane) 8 words
static constexpr uint32_t BT_FRAG_WORDS = 8;

// ---- inputs -> fragment table ------------------------------------------------------
// Element k = 32 blk + 16 s + 4 t + j of input row b (group b / 8, g = b % 8)
// lands in lane g*4 + t of group b / 8, word 4 s + (lo ? 2 : 0) + j / 2, half
// j % 2: the B fragment registers of mma m16n8k16 for K step s.
struct BatchPrepArgs {
    const float* x;           // [B][ldx] rows, or the embedding table when gather
    uint32_t ldx;
    uint32_t gather;          // row b = x + step[b].token * K
    const StepParams* step;   // [B]
    float* x_copy;            // non-null: raw rows copied here ([B][K], the residual stream)
    const float* norm_w;      // non-null: RMSNorm with these gains (upstream rmsnorm.c:15-92)
    float eps;
    uint32_t K, B, TG;        // TG: groups of 8 inputs in the table
    uint32_t* frag;           // [K/32][TG][32][8]
    float* tscale;            // [B]: 2^-e of the row
};

__device__ __forceinline__ int bt_exponent(float maxabs) {
    if (!(maxabs > 0.0f)) return 0;
    int E;
    frexpf(maxabs, &E);
    return min(max(15 - E, -100), 100);
}

// Grid (TG * 8 input rows, slices): every CTA of a row reads the whole row
// (its sum of squares and maximum are row-wide) and writes the fragments of
// its slice of the blocks; rows >= B write zeros.  The trigger comes first:
// the GEMV after it streams its weights meanwhile and waits for the whole
// grid before it reads a fragment.
__global__ void __launch_bounds__(256) batch_xprep_kernel(const BatchPrepArgs a) {
    extern __shared__ __align__(16) float brow[];
    __shared__ float s_red[8];
    __shared__ uint32_t s_max;
    const uint32_t b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = a.K, nb = K / 32;
    const uint32_t q0 = nb * 8 * blockIdx.y / gridDim.y, q1 = nb * 8 * (blockIdx.y + 1) / gridDim.y;
    pdl_trigger();
    pdl_wait();
    if (tid == 0) s_max = 0u;
    const bool live = b < a.B;
    float ss = 0.0f;
    if (live) {
        const float* src = a.gather ? a.x + (size_t)a.step[b].token * K : a.x + (size_t)b * a.ldx;
        for (uint32_t i = tid; i < K / 4; i += 256) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src) + i);
            reinterpret_cast<float4*>(brow)[i] = v;
            if (a.x_copy && blockIdx.y == 0) reinterpret_cast<float4*>(a.x_copy + (size_t)b * K)[i] = v;
            ss = __fmaf_rn(v.x, v.x, ss);
            ss = __fmaf_rn(v.y, v.y, ss);
            ss = __fmaf_rn(v.z, v.z, ss);
            ss = __fmaf_rn(v.w, v.w, ss);
        }
    }
    float r_norm = 1.0f;
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = 0; w < 8; ++w) tot += s_red[w];
        const float me = __fadd_rn(__fdiv_rn(tot, (float)K), a.eps);
        const float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
        const float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
        r_norm = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
    }
    __syncthreads();
    float mx = 0.0f;
    if (live)
        for (uint32_t k = tid; k < K; k += 256) {
            float v = brow[k];
            if (a.norm_w) v = __fmul_rn(__fmul_rn(v, r_norm), __ldg(a.norm_w + k));
            brow[k] = v;
            mx = fmaxf(mx, fabsf(v));
        }
    mx = warp_max(mx);
    if (lane == 0) atomicMax(&s_max, __float_as_uint(mx));
    __syncthreads();
    const int e = bt_exponent(__uint_as_float(s_max));
    const float mul = ldexpf(1.0f, e);
    if (tid == 0 && live && blockIdx.y == 0) a.tscale[b] = ldexpf(1.0f, -e);
    const uint32_t tg = b >> 3, g = b & 7;
    // thread: four consecutive k of one (block, step, t)
    for (uint32_t q = q0 + tid; q < q1; q += 256) {
        const uint32_t blk = q >> 3, st = (q >> 2) & 1, t = q & 3;
        const uint32_t k = blk * 32 + st * 16 + 4 * t;
        uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
        if (live) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const float v0 = brow[k + 2 * p] * mul, v1 = brow[k + 2 * p + 1] * mul;
                const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
                const __half l0 = __float2half_rn(v0 - __half2float(h0));
                const __half l1 = __float2half_rn(v1 - __half2float(h1));
                const __half2 hh = __halves2half2(h0, h1), ll = __halves2half2(l0, l1);
                hw[p] = *reinterpret_cast<const uint32_t*>(&hh);
                lw[p] = *reinterpret_cast<const uint32_t*>(&ll);
            }
        }
        uint32_t* dst = a.frag + (((size_t)blk * a.TG + tg) * 32 + g * 4 + t) * BT_FRAG_WORDS + st * 4;
        *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], lw[0], lw[1]);
    }
}

// ---- the batched GEMV ---------------------------------------------------------------
struct BatchGemvArgs {
    const uint8_t* w;        // slab tiles
    uint32_t M, K, n_slabs, nb;
    uint32_t B, TG;
    const uint32_t* frag;    // input fragments (batch_xprep_kernel)
    const float* tscale;     // [B]
    int epi;                 // GemvEpilogue
    float* y;                // [B][ldy]
    uint32_t ldy;
    const float* resid;      // EPI_RESID: [B][ldy] (may alias y)
    const StepParams* step;  // [B]: positions for EPI_QKV
    // EPI_QKV: q -> y (RoPE), k (RoPE) and v -> sequence b's cache at its pos
    const float* rope_cos;
    const float* rope_sin;
    float* kv;               // cache of sequence 0, this layer's plane [n_kv][max_seq][2 hd]
                             // (paged: the page pool, [page][n_layers][n_kv][page_rows][2 hd])
    size_t kv_seq_stride;    // floats from one sequence's cache to the next
    uint32_t hd, q_rows, kv_rows, max_seq;
    const uint32_t* pages;   // paged caches: [B][pages_per_seq] page of each page_rows rows
    uint32_t page_rows, pages_per_seq, n_layers, layer;
};

__device__ __forceinline__ uint32_t nib2h(uint32_t w, uint32_t sel) {
    // bytes (n0, n1) of w (values 0..15) -> fp16 pair (n0 - 8, n1 - 8), exact:
    // 0x6400 | n is 1024 + n, minus 1032
    const uint32_t r = __byte_perm(w, 0x64646464u, sel);
    __half2 h = *reinterpret_cast<const __half2*>(&r);
    h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Epilogue of one (row pair, input) of the pass: rows r0, r0 + 1 (global),
// values v0, v1 already scaled.
__device__ __forceinline__ void bt_epilogue(const BatchGemvArgs& a, uint32_t r0, uint32_t b, float v0, float v1) {
    float* yr = a.y + (size_t)b * a.ldy;
    if (a.epi == EPI_STORE || a.epi == EPI_RESID) {
        if (a.epi == EPI_RESID) {
            v0 = __fadd_rn(__ldcg(a.resid + (size_t)b * a.ldy + r0), v0);
            v1 = __fadd_rn(__ldcg(a.resid + (size_t)b * a.ldy + r0 + 1), v1);
        }
        yr[r0] = v0;
        if (r0 + 1 < a.M) yr[r0 + 1] = v1;
    } else if (a.epi == EPI_SILU) {
        yr[r0 / 2] = __fmul_rn(silu_poly(v0), v1);
    } else {  // EPI_QKV
        const uint32_t p = a.step[b].pos;
        const float* ct = a.rope_cos + (size_t)p * a.hd;
        const float* st = a.rope_sin + (size_t)p * a.hd;
        float o0, o1;
        // row p of head h in sequence b's cache
        auto row = [&](uint32_t h) -> float* {
            if (!a.pages) return a.kv + (size_t)b * a.kv_seq_stride + ((size_t)h * a.max_seq + p) * 2 * a.hd;
            const uint32_t pg = __ldg(a.pages + (size_t)b * a.pages_per_seq + p / a.page_rows);
            const uint32_t nkv = a.kv_rows / a.hd;
            return a.kv + ((((size_t)pg * a.n_layers + a.layer) * nkv + h) * a.page_rows + p % a.page_rows) * 2 * a.hd;
        };
        if (r0 < a.q_rows) {
            rope_pair(v0, v1, ct, st, r0 % a.hd, o0, o1);
            yr[r0] = o0;
            yr[r0 + 1] = o1;
        } else if (r0 < a.q_rows + a.kv_rows) {
            const uint32_t kr = r0 - a.q_rows, h = kr / a.hd, e = kr % a.hd;
            rope_pair(v0, v1, ct, st, e, o0, o1);
            float* dst = row(h) + e;
            dst[0] = o0;
            dst[1] = o1;
        } else {
            const uint32_t vr = r0 - a.q_rows - a.kv_rows, h = vr / a.hd, e = vr % a.hd;
            float* dst = row(h) + a.hd + e;
            dst[0] = v0;
            dst[1] = v1;
        }
    }
}

template <int TG>
__global__ void __launch_bounds__(BT_THREADS, 1) q4_batch_kernel(const BatchGemvArgs a) {
    extern __shared__ __align__(128) uint8_t bsm[];
    uint8_t* ring = bsm;
    float* red = reinterpret_cast<float*>(bsm + BT_STAGES * BT_STAGE_BYTES);  // [W][NS*32][16]
    __shared__ __align__(8) uint64_t full[BT_STAGES], empty[BT_STAGES];
    constexpr uint32_t NW = BT_WARPS, T = NW * 32;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x, cta = blockIdx.x;
    const uint32_t j0 = a.n_slabs * cta / G, j1 = a.n_slabs * (cta + 1) / G;
    const uint32_t nb = a.nb;
    const uint32_t n_bst = (nb + BT_SB - 1) / BT_SB;  // block stages per pass
    if (tid == 0) {
        for (uint32_t s = 0; s < BT_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == NW) {
        // ---- producer: per pass (<= 4 slabs), block stages; one bulk copy per slab ----
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t s = 0, ph = 0, k = 0;
            bool ok = true;
            for (uint32_t jp = j0; jp < j1 && ok; jp += BT_NS) {
                const uint32_t ns = min(BT_NS, j1 - jp);
                for (uint32_t bs = 0; bs < n_bst; ++bs, ++k) {
                    if (k >= BT_STAGES && !mbar_wait(&empty[s], ph ^ 1, QDEV_WAIT_EMPTY_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    const uint32_t b0 = bs * BT_SB, n = min(BT_SB, nb - b0);
                    mbar_arrive_expect_tx(&full[s], ns * n * GEMV_BLOCK_BYTES);
                    for (uint32_t i = 0; i < ns; ++i)
                        bulk_g2s(ring + (size_t)s * BT_STAGE_BYTES + (size_t)i * BT_SB * GEMV_BLOCK_BYTES,
                                 a.w + ((size_t)(jp + i) * nb + b0) * GEMV_BLOCK_BYTES, n * GEMV_BLOCK_BYTES,
                                 &full[s], pol);
                    if (++s == BT_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
        }
        pdl_wait();
        return;
    }

    // ---- consumers ----
    pdl_wait();
    const uint32_t g = lane >> 2, t = lane & 3;
    uint32_t s = 0, ph = 0;
    // input fragments of block blk: [TG][lane][8 words]; a warp takes blocks
    // warp, warp + NW, ... (BT_SB is a multiple of NW), so the next block's
    // fragments are loaded (from L2) while this one's MMAs run
    auto load_frag = [&](uint4 (&xf)[TG][2], uint32_t blk) {
#pragma unroll
        for (int q = 0; q < TG; ++q) {
            const uint4* src = reinterpret_cast<const uint4*>(a.frag + (((size_t)blk * a.TG + q) * 32 + lane) * BT_FRAG_WORDS);
            xf[q][0] = __ldcg(src);
            xf[q][1] = __ldcg(src + 1);
        }
    };
    static_assert(BT_SB % BT_WARPS == 0, "a warp's blocks follow one another across stages");
    for (uint32_t jp = j0; jp < j1; jp += BT_NS) {
        const uint32_t ns = min(BT_NS, j1 - jp);
        uint4 nxt[TG][2];
        if (warp < nb) load_frag(nxt, warp);
        float acc[BT_NS][2][TG][4];
#pragma unroll
        for (int i = 0; i < (int)BT_NS; ++i)
#pragma unroll
            for (int rg = 0; rg < 2; ++rg)
#pragma unroll
                for (int q = 0; q < TG; ++q)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[i][rg][q][e] = 0.0f;
        for (uint32_t bs = 0; bs < n_bst; ++bs) {
            mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
            const uint32_t b0 = bs * BT_SB, n = min(BT_SB, nb - b0);
            for (uint32_t bi = warp; bi < n; bi += NW) {
                const uint32_t blk = b0 + bi;
                uint4 xf[TG][2];
#pragma unroll
                for (int q = 0; q < TG; ++q) {
                    xf[q][0] = nxt[q][0];
                    xf[q][1] = nxt[q][1];
                }
                if (blk + NW < nb) load_frag(nxt, blk + NW);
#pragma unroll
                for (int i = 0; i < (int)BT_NS; ++i) {
                    if ((uint32_t)i >= ns) break;
                    const uint8_t* tile = ring + (size_t)s * BT_STAGE_BYTES + ((size_t)i * BT_SB + bi) * GEMV_BLOCK_BYTES;
                    const uint4 qv = *reinterpret_cast<const uint4*>(tile + lane * 16);
                    const float4 sc = *reinterpret_cast<const float4*>(tile + 512 + g * 16);
                    const uint32_t words[4] = {qv.x, qv.y, qv.z, qv.w};  // rows g, g+8, g+16, g+24
#pragma unroll
                    for (int rg = 0; rg < 2; ++rg) {
                        float d[TG][4];
#pragma unroll
                        for (int q = 0; q < TG; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.0f;
#pragma unroll
                        for (int st = 0; st < 2; ++st) {
                            const uint32_t wa = st ? (words[2 * rg] >> 4) & 0x0F0F0F0Fu : words[2 * rg] & 0x0F0F0F0Fu;
                            const uint32_t wb = st ? (words[2 * rg + 1] >> 4) & 0x0F0F0F0Fu : words[2 * rg + 1] & 0x0F0F0F0Fu;
                            const uint32_t a0 = nib2h(wa, 0x5140), a2 = nib2h(wa, 0x5342);
                            const uint32_t a1 = nib2h(wb, 0x5140), a3 = nib2h(wb, 0x5342);
#pragma unroll
                            for (int q = 0; q < TG; ++q) {
                                const uint4 f = xf[q][st];
                                mma_f16(d[q], a0, a1, a2, a3, f.x, f.y);  // hi
                                mma_f16(d[q], a0, a1, a2, a3, f.z, f.w);  // lo
                            }
                        }
                        const float s0 = rg ? sc.z : sc.x, s1 = rg ? sc.w : sc.y;  // rows g(+16), g+8(+16)
#pragma unroll
                        for (int q = 0; q < TG; ++q) {
                            acc[i][rg][q][0] = __fmaf_rn(s0, d[q][0], acc[i][rg][q][0]);
                            acc[i][rg][q][1] = __fmaf_rn(s0, d[q][1], acc[i][rg][q][1]);
                            acc[i][rg][q][2] = __fmaf_rn(s1, d[q][2], acc[i][rg][q][2]);
                            acc[i][rg][q][3] = __fmaf_rn(s1, d[q][3], acc[i][rg][q][3]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == BT_STAGES) {
                s = 0;
                ph ^= 1;
            }
        }
        // ---- reduce the warps' partial sums, then the epilogue ----
        // D fragment of (rg, q): rows g + 16 rg (+8 for e >= 2), inputs 8 q + 2 t + (e & 1)
#pragma unroll
        for (int i = 0; i < (int)BT_NS; ++i)
#pragma unroll
            for (int rg = 0; rg < 2; ++rg)
#pragma unroll
                for (int q = 0; q < TG; ++q)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t row = i * 32 + g + 16 * rg + (e >= 2 ? 8 : 0);
                        const uint32_t col = 8 * q + 2 * t + (e & 1);
                        red[((size_t)warp * BT_NS * 32 + row) * BT_MAXB + col] = acc[i][rg][q][e];
                    }
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        const uint32_t B = a.B;
        for (uint32_t idx = tid; idx < ns * 16 * B; idx += T) {
            const uint32_t pr = idx / B, b = idx % B;  // row pair within the pass, input
            float v0 = 0.0f, v1 = 0.0f;
            for (uint32_t w = 0; w < NW; ++w) {
                v0 += red[((size_t)w * BT_NS * 32 + 2 * pr) * BT_MAXB + b];
                v1 += red[((size_t)w * BT_NS * 32 + 2 * pr + 1) * BT_MAXB + b];
            }
            const float ts = __ldg(a.tscale + b);
            const uint32_t r0 = jp * 32 + 2 * pr;
            if (r0 < a.M) bt_epilogue(a, r0, b, v0 * ts, v1 * ts);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(T));  // red[] free for the next pass
    }
}

// ---- the batched LM head --------------------------------------------------------------
// logits[b][v] = W_out[v] . RMSNorm(x_b) for B inputs, the argmax key of
// every input folded in.  W_out is fp32 [V][K]: a warp takes 16-row groups,
// splits each row block into fp16 hi + lo after a power-of-two scale of the
// whole matrix (wexp, computed at set-up) and multiplies with the inputs'
// hi + lo fragments (the three products hi*hi, hi*lo, lo*hi per K step,
// every product exact, fp32 accumulation promoted into registers every 32 K).
struct BatchHeadArgs {
    const float* w;          // [V][K]: this rank's vocabulary rows under tensor parallelism
    uint32_t V, K, B, TG;
    uint32_t row_base;       // global index of row 0 (vocabulary split)
    uint32_t ldl;            // logits row stride (>= V)
    float wmul, wdiv;        // 2^wexp, 2^-wexp
    const uint32_t* frag;    // normalized inputs, batch_xprep_kernel layout
    const float* tscale;     // [B]
    float* logits;           // [B][ldl]
    unsigned long long* best;  // [B] argmax keys
};

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
    __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int TG>
__global__ void __launch_bounds__(256) batch_head_kernel(const BatchHeadArgs a) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3;
    const uint32_t n_groups = (a.V + 15) / 16, nb = a.K / 32;
    const uint32_t gw = blockIdx.x * 8 + warp, nw = gridDim.x * 8;
    pdl_wait();
    __shared__ unsigned long long s_best[BT_MAXB];
    if (threadIdx.x < BT_MAXB) s_best[threadIdx.x] = 0ull;
    __syncthreads();
    for (uint32_t grp = gw; grp < n_groups; grp += nw) {
        const uint32_t ra = grp * 16 + g, rb = ra + 8;
        const float* wa = a.w + (size_t)min(ra, a.V - 1) * a.K;
        const float* wb = a.w + (size_t)min(rb, a.V - 1) * a.K;
        float acc[TG][4];
#pragma unroll
        for (int q = 0; q < TG; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.0f;
        // W of blocks blk + 1 and blk + 2 are in flight while block blk is
        // multiplied (two blocks ahead: a warp walks its rows block by block,
        // so the loads in flight per warp set the bandwidth)
        float4 cur[2][2], nxt[2][2], nx2[2][2];
        auto load_w = [&](float4 (&dst)[2][2], uint32_t blk) {
#pragma unroll
            for (int st = 0; st < 2; ++st) {
                const uint32_t k = blk * 32 + st * 16 + 4 * t;
                dst[st][0] = ldg_stream_f4(reinterpret_cast<const float4*>(wa + k));
                dst[st][1] = ldg_stream_f4(reinterpret_cast<const float4*>(wb + k));
            }
        };
        // the inputs' fragments of block blk + 1 are requested with them
        auto load_x = [&](uint4 (&dst)[TG][2], uint32_t blk) {
#pragma unroll
            for (int q = 0; q < TG; ++q) {
                const uint4* src = reinterpret_cast<const uint4*>(a.frag + (((size_t)blk * a.TG + q) * 32 + lane) * BT_FRAG_WORDS);
                dst[q][0] = __ldcg(src);
                dst[q][1] = __ldcg(src + 1);
            }
        };
        uint4 xnext[TG][2];
        load_w(cur, 0);
        if (nb > 1) load_w(nxt, 1);
        load_x(xnext, 0);
        for (uint32_t blk = 0; blk < nb; ++blk) {
            if (blk + 2 < nb) load_w(nx2, blk + 2);
            uint4 xf[TG][2];
#pragma unroll
            for (int q = 0; q < TG; ++q) {
                xf[q][0] = xnext[q][0];
                xf[q][1] = xnext[q][1];
            }
            if (blk + 1 < nb) load_x(xnext, blk + 1);
            float d[TG][4];
#pragma unroll
            for (int q = 0; q < TG; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.0f;
#pragma unroll
            for (int st = 0; st < 2; ++st) {
                const float4 va = cur[st][0], vb = cur[st][1];
                // A: a0 = row g (k, k+1), a1 = row g+8 (k, k+1), a2 = row g (k+2, k+3), a3 = row g+8 (k+2, k+3)
                const float src[4][2] = {{va.x * a.wmul, va.y * a.wmul}, {vb.x * a.wmul, vb.y * a.wmul},
                                         {va.z * a.wmul, va.w * a.wmul}, {vb.z * a.wmul, vb.w * a.wmul}};
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const __half2 h = __floats2half2_rn(src[r][0], src[r][1]);
                    const float2 hf = __half22float2(h);
                    hi[r] = *reinterpret_cast<const uint32_t*>(&h);
                    lo[r] = pack_h2(src[r][0] - hf.x, src[r][1] - hf.y);
                }
#pragma unroll
                for (int q = 0; q < TG; ++q) {
                    const uint4 f = xf[q][st];
                    mma_f16(d[q], hi[0], hi[1], hi[2], hi[3], f.x, f.y);
                    mma_f16(d[q], hi[0], hi[1], hi[2], hi[3], f.z, f.w);
                    mma_f16(d[q], lo[0], lo[1], lo[2], lo[3], f.x, f.y);
                }
            }
#pragma unroll
            for (int q = 0; q < TG; ++q)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[q][e] = __fadd_rn(acc[q][e], d[q][e]);
#pragma unroll
            for (int st = 0; st < 2; ++st) {
                cur[st][0] = nxt[st][0];
                cur[st][1] = nxt[st][1];
                nxt[st][0] = nx2[st][0];
                nxt[st][1] = nx2[st][1];
            }
        }
        // D: rows g (e < 2) / g + 8, inputs 8 q + 2 t + (e & 1)
#pragma unroll
        for (int q = 0; q < TG; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t b = 8 * q + 2 * t + (e & 1), row = e < 2 ? ra : rb;
                if (b >= a.B || row >= a.V) continue;
                const float v = acc[q][e] * a.wdiv * __ldg(a.tscale + b);
                a.logits[(size_t)b * a.ldl + row] = v;
                // order-preserving key, lowest index wins ties (upstream main.c:870-881)
                const uint32_t u = __float_as_uint(v);
                const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
                atomicMax(&s_best[b], ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (a.row_base + row)));
            }
    }
    __syncthreads();
    if (threadIdx.x < a.B && s_best[threadIdx.x]) atomicMax(&a.best[threadIdx.x], s_best[threadIdx.x]);
}

// Every sequence: publish its argmax token, advance its position.
struct BatchAdvanceArgs {
    StepParams* step;          // [B]
    unsigned long long* best;  // [B]
    uint32_t* token_out;       // [cap][B]
    uint32_t* token_count;
    uint32_t token_cap, B;
};

__global__ void batch_advance_kernel(const BatchAdvanceArgs a) {
    pdl_wait();
    const uint32_t b = threadIdx.x;
    const uint32_t n = *a.token_count;
    __syncthreads();
    if (b < a.B) {
        const unsigned long long k = a.best[b];
        const uint32_t tok = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
        if (n < a.token_cap) a.token_out[(size_t)n * a.B + b] = tok;
        StepParams s = a.step[b];
        s.token = tok;
        s.pos = s.pos + 1;
        s.n_row = s.pos + 1;
        s.valid = s.pos + 1;
        a.step[b] = s;
        a.best[b] = 0ull;
    }
    __syncthreads();
    if (b == 0) *a.token_count = n + 1;
}

}  // namespace qb200
