// prefill.cuh — prompt processing (seq_len > 1) on the Blackwell tensor cores.
//
// Upstream runs a prompt row by row: llama_forward (src/models/model.c:
// 1120-1165) calls q_gemv_q4_f32_avx2 (src/ops/avx2/matmul.c:98-271) once per
// row and projection, then attention over the causal rows (model.c:1366-1422,
// src/ops/avx2/causal_mask_fp32.c:16-138, softmax.c:17-132).  Here every
// projection of a layer is ONE dense contraction Y[S][M] = X[S][K] W[M][K]^T
// on tcgen05.mma (TMA-fed shared-memory operands, fp32 accumulators in TMEM).
//
// Precision.  The per-kernel bar is 1e-4 relative; rounding the activations
// to bf16 (8 bits) would miss it by ~40x.  So each operand is carried as two
// fp16 halves, v = hi + lo (hi = fp16(v), lo = fp16(v - hi): 22 significant
// bits), after scaling it by a power of two into fp16's range (per token row
// for X, per weight row for W; the epilogue multiplies the scales back, which
// is exact).  Three MMAs per K-step, hi*hi + hi*lo + lo*hi, accumulate in
// fp32; the dropped lo*lo term is ~2^-22 relative.  The products of fp16
// operands are exact in fp32, so the result is an fp32 dot product with a
// different summation order than upstream's — inside the bar.
//
// Kernels:
//   w_split_kernel     Q4_0 slab tiles -> W_hi, W_lo [M][K] fp16 + row scales
//   act_split_kernel   X rows (optional embedding gather, RMSNorm) -> X_hi,
//                      X_lo [S][K] fp16 + token scales
//   pf_gemm_kernel     persistent tcgen05 GEMM with the decode epilogues
//                      (store, residual add, SiLU*up, RoPE + KV store)
//   attn_prefill_kernel  causal GQA attention, two passes (row max, then the
//                      upstream polynomial-exp softmax and P.V)
#pragma once

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

// ---- tile shape -------------------------------------------------------------------
static constexpr uint32_t PF_BM = 128;  // token rows per tile (MMA M = TMEM lanes)
static constexpr uint32_t PF_BN = 128;  // weight rows per tile (MMA N = accumulator columns)
static constexpr uint32_t PF_BK = 64;   // fp16 per K chunk: one 128-byte swizzle row
static constexpr uint32_t PF_STAGES = 3;
static constexpr uint32_t PF_A_BYTES = PF_BM * PF_BK * 2;                    // 16 KB
static constexpr uint32_t PF_B_BYTES = PF_BN * PF_BK * 2;                    // 16 KB
static constexpr uint32_t PF_STAGE_BYTES = 2 * PF_A_BYTES + 2 * PF_B_BYTES;  // hi + lo of each
static constexpr uint32_t PF_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
// The tensor core adds each MMA's products into its fp32 accumulator with
// truncation toward zero at the accumulator's precision, so the error grows
// with the number of MMAs per accumulation (measured: 3e-4 relative at
// K = 14336 in one accumulator, 9e-6 with the fold every 4 chunks).  So the MMAs accumulate PF_SEG K chunks (48 MMAs) into
// one of two partial buffers and the epilogue warps add each partial, in
// correctly rounded fp32, into a running sum kept in TMEM:
// columns [0, N) and [N, 2N) partials, [2N, 3N) the running sum.
static constexpr uint32_t PF_SEG = 4;
static constexpr uint32_t PF_TMEM_COLS = 512;
static constexpr size_t PF_SMEM = (size_t)PF_STAGES * PF_STAGE_BYTES + 1024 /*align*/ + 256;

// fp16 range scaling: a row is multiplied by 2^e with e chosen so its largest
// magnitude lands in [2^14, 2^15) (fp16 max 65504).
__device__ __forceinline__ int pf_exponent(float maxabs) {
    if (!(maxabs > 0.0f)) return 0;
    int E;
    frexpf(maxabs, &E);  // maxabs = f 2^E, f in [0.5, 1)
    return min(max(15 - E, -100), 100);
}

__device__ __forceinline__ void pf_split(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// ---- weights: slab tiles -> fp16 halves ---------------------------------------------
// One CTA per 32-row slab (the decode layout of gemv_q4.cuh).  Pass 1 finds
// each row's largest scale; pass 2 decodes (q - 8) * s in fp32 (the value
// upstream's block decode forms), scales it by the row's power of two and
// writes hi and lo rows through a shared-memory transpose (coalesced rows).
__global__ void __launch_bounds__(256) w_split_kernel(const uint8_t* __restrict__ packed, uint32_t M,
                                                      uint32_t nb, __half* __restrict__ whi,
                                                      __half* __restrict__ wlo, float* __restrict__ rscale) {
    __shared__ uint32_t s_max[32];
    __shared__ float s_mul[32];
    __shared__ float tile[8][32][33];
    const uint32_t j = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = nb * 32;
    const uint8_t* slab = packed + (size_t)j * nb * GEMV_BLOCK_BYTES;
    if (tid < 32) s_max[tid] = 0u;
    __syncthreads();
    for (uint32_t e = tid; e < nb * 32; e += 256) {
        const uint32_t b = e >> 5, r = e & 31;
        const float sc = *reinterpret_cast<const float*>(slab + (size_t)b * GEMV_BLOCK_BYTES + 512 +
                                                          ((r & 7) * 4 + (r >> 3)) * 4);
        atomicMax(&s_max[r], __float_as_uint(fabsf(sc)));
    }
    __syncthreads();
    if (tid < 32) {
        const int e = pf_exponent(8.0f * __uint_as_float(s_max[tid]));
        s_mul[tid] = ldexpf(1.0f, e);
        const uint32_t row = j * 32 + tid;
        if (row < M) rscale[row] = ldexpf(1.0f, -e);
    }
    __syncthreads();
    const uint32_t g = lane >> 2, t = lane & 3;
    for (uint32_t b = warp; b < nb; b += 8) {
        const uint8_t* blk = slab + (size_t)b * GEMV_BLOCK_BYTES;
        const uint4 q = *reinterpret_cast<const uint4*>(blk + lane * 16);
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
            const uint32_t r = g + 8 * qd;
            const float s = *reinterpret_cast<const float*>(blk + 512 + (g * 4 + qd) * 4);
#pragma unroll
            for (int by = 0; by < 4; ++by) {
                const uint32_t byte = (words[qd] >> (8 * by)) & 0xFFu;
                tile[warp][r][4 * t + by] = __fmul_rn((float)((int)(byte & 15u) - 8), s);
                tile[warp][r][16 + 4 * t + by] = __fmul_rn((float)((int)(byte >> 4) - 8), s);
            }
        }
        __syncwarp();
        // lanes 0..15 write row r, lanes 16..31 row r + 1: 32 fp16 = 64 bytes each
        const uint32_t half = lane >> 4, c = (lane & 15) * 2;
        for (uint32_t r = half; r < 32; r += 2) {
            const uint32_t row = j * 32 + r;
            const float m = s_mul[r];
            __half h0, l0, h1, l1;
            pf_split(tile[warp][r][c] * m, h0, l0);
            pf_split(tile[warp][r][c + 1] * m, h1, l1);
            if (row < M) {
                const size_t o = (size_t)row * K + b * 32 + c;
                *reinterpret_cast<__half2*>(whi + o) = __halves2half2(h0, h1);
                *reinterpret_cast<__half2*>(wlo + o) = __halves2half2(l0, l1);
            }
        }
        __syncwarp();
    }
}

// ---- activations: rows -> fp16 halves -------------------------------------------------
struct ActSplitArgs {
    const float* x;          // [S][ldx] fp32, or the embedding table when tokens != null
    const uint32_t* tokens;  // non-null: row t = x + tokens[t] * K (embedding gather)
    uint32_t ldx;
    float* x_copy;           // non-null: raw row t copied to x_copy + t * K (residual stream)
    const float* norm_w;     // non-null: RMSNorm with these gains (upstream rmsnorm.c:15-92)
    float eps;
    uint32_t K;
    __half* hi;              // [S][K]
    __half* lo;
    float* tscale;           // [S]: 2^-e of the row
};

// One CTA per row; the row is staged in shared memory (K floats).
__global__ void __launch_bounds__(256) act_split_kernel(const ActSplitArgs a) {
    extern __shared__ __align__(16) float row[];
    __shared__ float s_red[8];
    __shared__ uint32_t s_max;
    const uint32_t t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = a.K, n4 = K / 4;
    const float* src = a.tokens ? a.x + (size_t)a.tokens[t] * K : a.x + (size_t)t * a.ldx;
    float ss = 0.0f;
    for (uint32_t i = tid; i < n4; i += 256) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src) + i);
        reinterpret_cast<float4*>(row)[i] = v;
        if (a.x_copy) reinterpret_cast<float4*>(a.x_copy + (size_t)t * K)[i] = v;
        ss = __fmaf_rn(v.x, v.x, ss);
        ss = __fmaf_rn(v.y, v.y, ss);
        ss = __fmaf_rn(v.z, v.z, ss);
        ss = __fmaf_rn(v.w, v.w, ss);
    }
    if (tid == 0) s_max = 0u;
    float r_norm = 1.0f;
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = 0; w < 8; ++w) tot += s_red[w];
        // upstream rmsnorm.c: mean of squares + eps, rsqrt + one Newton step
        const float me = __fadd_rn(__fdiv_rn(tot, (float)K), a.eps);
        const float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
        const float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
        r_norm = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
    }
    __syncthreads();
    float mx = 0.0f;
    for (uint32_t k = tid; k < K; k += 256) {
        float v = row[k];
        if (a.norm_w) v = __fmul_rn(__fmul_rn(v, r_norm), __ldg(a.norm_w + k));
        row[k] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    mx = warp_max(mx);
    if (lane == 0) atomicMax(&s_max, __float_as_uint(mx));
    __syncthreads();
    const int e = pf_exponent(__uint_as_float(s_max));
    const float mul = ldexpf(1.0f, e);
    if (tid == 0) a.tscale[t] = ldexpf(1.0f, -e);
    for (uint32_t k = 2 * tid; k < K; k += 512) {
        __half h0, l0, h1, l1;
        pf_split(row[k] * mul, h0, l0);
        pf_split(row[k + 1] * mul, h1, l1);
        const size_t o = (size_t)t * K + k;
        *reinterpret_cast<__half2*>(a.hi + o) = __halves2half2(h0, h1);
        *reinterpret_cast<__half2*>(a.lo + o) = __halves2half2(l0, l1);
    }
}

// ---- tcgen05 helpers (inline PTX) ----------------------------------------------------

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout TMA writes (rows of 128 bytes, 8-row groups 1024 bytes apart; the
// tile base 1024-byte aligned).  LBO is unused for this layout (1), SBO =
// 1024 bytes, version 1 (sm_100), layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D f32, A and B f16, both K-major,
// N = PF_BN, M = PF_BM.
static constexpr uint32_t PF_IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((PF_BN >> 3) << 17) |
                                     ((PF_BM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc,
                                         uint32_t idesc = PF_IDESC) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_3d_pf(void* dst_smem, const CUtensorMap* map, int x, int y, int z,
                                               uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst_smem)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// ---- the GEMM -------------------------------------------------------------------------
struct PfGemmArgs {
    uint32_t S, M, K;          // token rows, weight rows, reduction length
    uint32_t n_mt, n_nt;       // token tiles, weight-row tiles
    const float* tscale;       // [S] 2^-e per token row
    const float* rscale;       // [M] 2^-e per weight row
    int epi;                   // GemvEpilogue
    float* y;                  // output rows, stride ldy floats
    uint32_t ldy;
    const float* resid;        // EPI_RESID: [S][ldy] (may alias y)
    // EPI_QKV: columns [q | k | v]; q -> y (RoPE), k (RoPE) and v -> the cache
    const float* rope_cos;
    const float* rope_sin;
    float* kv_layer;           // [n_kv][max_seq][2 hd] of this layer
    uint32_t hd, q_rows, kv_rows, max_seq, pos;
};

// Epilogue of 32 accumulator columns n0..n0+31 of token row `tok` (one
// thread = one token row; column pairs sit in the same thread).
__device__ __forceinline__ void pf_epilogue32(const PfGemmArgs& a, uint32_t tok, uint32_t n0, float tsc,
                                              float (&v)[32]) {
    if (tok >= a.S || n0 >= a.M) return;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = v[i] * tsc * __ldg(a.rscale + min(n0 + i, a.M - 1));
    const uint32_t nn = min(32u, a.M - n0);
    float* yr = a.y + (size_t)tok * a.ldy;
    if (a.epi == EPI_STORE || a.epi == EPI_RESID) {
        if (nn == 32 && (a.ldy % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                if (a.epi == EPI_RESID) {
                    const float4 r = __ldcg(reinterpret_cast<const float4*>(a.resid + (size_t)tok * a.ldy + n0 + i));
                    o = make_float4(__fadd_rn(r.x, o.x), __fadd_rn(r.y, o.y), __fadd_rn(r.z, o.z),
                                    __fadd_rn(r.w, o.w));
                }
                *reinterpret_cast<float4*>(yr + n0 + i) = o;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if ((uint32_t)i < nn)
                    yr[n0 + i] = a.epi == EPI_RESID ? __fadd_rn(a.resid[(size_t)tok * a.ldy + n0 + i], v[i]) : v[i];
        }
    } else if (a.epi == EPI_SILU) {
        // interleaved (gate_i, up_i) columns: upstream silu.c (poly exp) then mul_fp32.c
#pragma unroll
        for (int i = 0; i < 32; i += 2)
            if ((uint32_t)i < nn) yr[(n0 + i) / 2] = __fmul_rn(silu_poly(v[i]), v[i + 1]);
    } else {  // EPI_QKV: a 32-column group lies inside one of q, k, v (hd % 32 == 0)
        const uint32_t p = a.pos + tok;
        const float* ct = a.rope_cos + (size_t)p * a.hd;
        const float* st = a.rope_sin + (size_t)p * a.hd;
        if (n0 < a.q_rows) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                float o0, o1;
                rope_pair(v[i], v[i + 1], ct, st, (n0 + i) % a.hd, o0, o1);
                yr[n0 + i] = o0;
                yr[n0 + i + 1] = o1;
            }
        } else if (n0 < a.q_rows + a.kv_rows) {
            const uint32_t kr = n0 - a.q_rows, h = kr / a.hd, e0 = kr % a.hd;
            float* dst = a.kv_layer + ((size_t)h * a.max_seq + p) * 2 * a.hd + e0;
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                float o0, o1;
                rope_pair(v[i], v[i + 1], ct, st, e0 + i, o0, o1);
                dst[i] = o0;
                dst[i + 1] = o1;
            }
        } else {
            const uint32_t vr = n0 - a.q_rows - a.kv_rows, h = vr / a.hd, e0 = vr % a.hd;
            float* dst = a.kv_layer + ((size_t)h * a.max_seq + p) * 2 * a.hd + a.hd + e0;
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
    }
}

// Persistent: CTA c takes tiles c, c + grid, ...; tile t = (weight tile
// t / n_mt, token tile t % n_mt), so CTAs running at once share weight tiles
// (read from HBM once, then from L2).  Roles: warp 0 lane 0 issues the TMA
// loads of a 3-stage ring (A_hi, A_lo, B_hi, B_lo per stage); warp 1 owns
// TMEM and its lane 0 issues the MMAs, PF_SEG K chunks per partial buffer
// (alternating between two, so the MMAs run on while the previous partial is
// folded); warps 2..5 (TMEM lanes 32 (w % 4) + i) fold each partial into the
// running sum and, after a tile's last partial, run the epilogue.  Every
// wait is bounded; a role that gives up records the code and stops, the
// others then time out too, and the MMA issuer drains its MMAs before TMEM
// is freed.
__global__ void __launch_bounds__(PF_THREADS, 1)
    pf_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const PfGemmArgs a) {
    extern __shared__ uint8_t pf_smem_raw[];
    const uint32_t base = (smem_u32(pf_smem_raw) + 1023u) & ~1023u;
    uint8_t* smem = pf_smem_raw + (base - smem_u32(pf_smem_raw));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + PF_STAGES * PF_STAGE_BYTES);
    uint64_t* empty = full + PF_STAGES;
    uint64_t* pfull = empty + PF_STAGES;
    uint64_t* pfree = pfull + 2;
    uint64_t* drain = pfree + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n_tiles = a.n_mt * a.n_nt;
    const uint32_t nk = (a.K + PF_BK - 1) / PF_BK;
    constexpr uint32_t SEG = PF_SEG;
    const uint32_t nseg = (nk + SEG - 1) / SEG;

    if (tid == 0) {
        for (uint32_t s = 0; s < PF_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&pfull[b], 1);
            mbar_init(&pfree[b], 4);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(PF_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            uint32_t s = 0, ph = 0, issued = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const int mt = (int)(t % a.n_mt), nt = (int)(t / a.n_mt);
                for (uint32_t kc = 0; kc < nk; ++kc) {
                    if (issued >= PF_STAGES && !mbar_wait(&empty[s], ph ^ 1, QDEV_WAIT_EMPTY_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + (size_t)s * PF_STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], PF_STAGE_BYTES);
                    const int kx = (int)(kc * PF_BK);
                    tma_load_3d_pf(st, &map_a, kx, mt * (int)PF_BM, 0, &full[s]);
                    tma_load_3d_pf(st + PF_A_BYTES, &map_a, kx, mt * (int)PF_BM, 1, &full[s]);
                    tma_load_3d_pf(st + 2 * PF_A_BYTES, &map_b, kx, nt * (int)PF_BN, 0, &full[s]);
                    tma_load_3d_pf(st + 2 * PF_A_BYTES + PF_B_BYTES, &map_b, kx, nt * (int)PF_BN, 1, &full[s]);
                    ++issued;
                    if (++s == PF_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            if (!ok) {
                // wait (bounded) for the copies still in flight into the ring
                for (uint32_t i = 0; i < PF_STAGES && i < issued; ++i) {
                    if (s == 0) {
                        s = PF_STAGES;
                        ph ^= 1;
                    }
                    --s;
                    mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            uint32_t s = 0, ph = 0, g = 0;  // ring slot, parity, partials started
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                for (uint32_t kc = 0; kc < nk && ok; ++kc) {
                    const uint32_t buf = g & 1;
                    if (kc % SEG == 0) {
                        if (g >= 2 && !mbar_wait(&pfree[buf], ((g >> 1) - 1) & 1, QDEV_WAIT_EMPTY_TIMEOUT)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    if (!mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + buf * PF_BN;
                    const uint32_t st = base + s * PF_STAGE_BYTES;
#pragma unroll
                    for (uint32_t kk = 0; kk < PF_BK / 16; ++kk) {
                        const uint64_t ahi = umma_desc_sw128(st + kk * 32);
                        const uint64_t alo = umma_desc_sw128(st + PF_A_BYTES + kk * 32);
                        const uint64_t bhi = umma_desc_sw128(st + 2 * PF_A_BYTES + kk * 32);
                        const uint64_t blo = umma_desc_sw128(st + 2 * PF_A_BYTES + PF_B_BYTES + kk * 32);
                        umma_f16(d, ahi, bhi, ((kc % SEG) | kk) != 0);
                        umma_f16(d, ahi, blo, 1);
                        umma_f16(d, alo, bhi, 1);
                    }
                    umma_commit(&empty[s]);  // the stage is free once these MMAs finish
                    if (++s == PF_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                    if (kc % SEG == SEG - 1 || kc == nk - 1) {
                        umma_commit(&pfull[buf]);  // this partial is complete
                        ++g;
                    }
                }
            }
            // every MMA issued has finished before TMEM can be freed
            umma_commit(drain);
            mbar_wait(drain, 0, QDEV_WAIT_FULL_TIMEOUT);
        }
    } else {
        // ---- fold + epilogue: warps 2..5, TMEM lane quarter warp % 4 ----
        const uint32_t quarter = warp & 3;
        const uint32_t lanes = (quarter * 32u) << 16;
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            const uint32_t mt = t % a.n_mt, nt = t / a.n_mt;
            const uint32_t tok = mt * PF_BM + quarter * 32 + lane;
            const float tsc = tok < a.S ? __ldg(a.tscale + tok) : 0.0f;
            for (uint32_t sg = 0; sg < nseg; ++sg, ++g) {
                const uint32_t buf = g & 1;
                if (!mbar_wait(&pfull[buf], (g >> 1) & 1, QDEV_WAIT_FULL_TIMEOUT)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t pa = tmem + lanes + buf * PF_BN, ra = tmem + lanes + 2 * PF_BN;
#pragma unroll 1
                for (uint32_t c = 0; c < PF_BN / 32; ++c) {
                    float v[32];
                    tmem_ld32(pa + c * 32, v);
                    if (sg > 0) {
                        float r[32];
                        tmem_ld32(ra + c * 32, r);
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(r[i], v[i]);
                    }
                    if (sg + 1 < nseg)
                        tmem_st32(ra + c * 32, v);
                    else
                        pf_epilogue32(a, tok, nt * PF_BN + c * 32, tsc, v);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&pfree[buf]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS)
                     : "memory");
    }
}

// ---- causal attention over the cache ------------------------------------------------
// Row t of the call (absolute position pos + t) attends to cache positions
// 0..pos+t (the causal mask of upstream causal_mask_fp32.c gives -1e9 to the
// rest, whose exponentials are exactly 0).  Softmax as upstream softmax.c
// over the row length N = pos + S: the maximum first, then the clamped
// polynomial exp on positions i < 8 floor(N/8) and expf on the tail, the sum,
// and P.V scaled by 1/sum.  The polynomial is not multiplicative, so no
// online rescaling: pass 1 finds each query's row maximum, pass 2 recomputes
// the scores and forms the exponentials against it.
//
// CTA = (KV head h, PF_AQ consecutive rows): its G query heads x PF_AQ rows
// make 64 query vectors sharing one stream of K/V chunks of 64 positions.
// Thread (qi, kj): 4 query vectors x 4 keys of a chunk for the scores, 4 query
// vectors x 8 head dims of the output.
static constexpr uint32_t PF_ATT_Q = 64;        // query vectors per CTA
static constexpr uint32_t PF_ATT_KC = 64;       // keys per chunk
static constexpr uint32_t PF_ATT_THREADS = 256;
static constexpr uint32_t PF_ATT_PAD = 68;      // padded row of the transposed tiles (floats)

struct PfAttnArgs {
    const float* q;       // [S][n_heads * hd] rotated queries
    const float* kv;      // this layer's cache [n_kv][max_seq][2 hd]
    float* out;           // [S][n_heads * hd]
    uint32_t S, pos, n_heads, n_kv, max_seq;
    float scale;
};

__host__ __device__ inline size_t pf_attn_smem(uint32_t hd) {
    // Q^T [hd][PAD] | K^T [hd][PAD] | V [KC][hd] | P^T [KC][PAD] | row stats
    return ((size_t)hd * PF_ATT_PAD * 2 + (size_t)PF_ATT_KC * hd + (size_t)PF_ATT_KC * PF_ATT_PAD +
            PF_ATT_Q * 16 * 2 + PF_ATT_Q * 2) * 4;
}

template <int HD, int G>
__global__ void __launch_bounds__(PF_ATT_THREADS) attn_prefill_kernel(const PfAttnArgs a) {
    static_assert(PF_ATT_Q % G == 0, "query vectors per CTA");
    constexpr uint32_t RQ = PF_ATT_Q / G;  // rows of the call per CTA
    extern __shared__ __align__(16) float sm[];
    float* qT = sm;                                   // [HD][PAD]: qT[d][v]
    float* kT = qT + HD * PF_ATT_PAD;                 // [HD][PAD]: kT[d][j]
    float* vs = kT + HD * PF_ATT_PAD;                 // [KC][HD]
    float* pT = vs + PF_ATT_KC * HD;                  // [KC][PAD]: pT[j][v]
    float* red = pT + PF_ATT_KC * PF_ATT_PAD;         // [Q][16] partial maxima / sums
    float* red2 = red + PF_ATT_Q * 16;
    float* rmax = red2 + PF_ATT_Q * 16;               // [Q]
    float* rinv = rmax + PF_ATT_Q;                    // [Q]
    const uint32_t tid = threadIdx.x;
    const uint32_t h = blockIdx.y, r0 = blockIdx.x * RQ;
    const uint32_t D = a.n_heads * HD;
    // query vector v = (row r0 + v / G, head h*G + v % G)
    for (uint32_t i = tid; i < PF_ATT_Q * (HD / 4); i += PF_ATT_THREADS) {
        const uint32_t v = i / (HD / 4), c = i % (HD / 4);
        const uint32_t row = r0 + v / G;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < a.S) x = __ldg(reinterpret_cast<const float4*>(a.q + (size_t)row * D + (h * G + v % G) * HD) + c);
        qT[(4 * c + 0) * PF_ATT_PAD + v] = x.x;
        qT[(4 * c + 1) * PF_ATT_PAD + v] = x.y;
        qT[(4 * c + 2) * PF_ATT_PAD + v] = x.z;
        qT[(4 * c + 3) * PF_ATT_PAD + v] = x.w;
    }
    const float* head = a.kv + (size_t)h * a.max_seq * 2 * HD;
    const uint32_t N = a.pos + a.S;        // upstream softmax row length of this call
    const uint32_t nv = N / 8 * 8;         // polynomial exp below nv, expf from nv on
    const uint32_t last_row = min(a.S, r0 + RQ) - 1;
    const uint32_t n_keys = a.pos + last_row + 1;  // keys any row of this CTA sees
    const uint32_t qi = tid / 16, kj = tid % 16;   // scores: vectors 4qi..+3, keys 4kj..+3
    uint32_t my_last[4];                           // last visible key of each of my vectors
#pragma unroll
    for (int u = 0; u < 4; ++u) my_last[u] = a.pos + r0 + (4 * qi + u) / G;

    auto load_k = [&](uint32_t k0) {
        for (uint32_t i = tid; i < PF_ATT_KC * (HD / 4); i += PF_ATT_THREADS) {
            const uint32_t j = i % PF_ATT_KC, c = i / PF_ATT_KC;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + j < n_keys) x = __ldg(reinterpret_cast<const float4*>(head + (size_t)(k0 + j) * 2 * HD) + c);
            kT[(4 * c + 0) * PF_ATT_PAD + j] = x.x;
            kT[(4 * c + 1) * PF_ATT_PAD + j] = x.y;
            kT[(4 * c + 2) * PF_ATT_PAD + j] = x.z;
            kT[(4 * c + 3) * PF_ATT_PAD + j] = x.w;
        }
    };
    auto scores = [&](float (&s)[4][4]) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < 4; ++w) s[u][w] = 0.0f;
#pragma unroll 8
        for (uint32_t d = 0; d < HD; ++d) {
            const float4 qv = *reinterpret_cast<const float4*>(qT + d * PF_ATT_PAD + 4 * qi);
            const float4 kv = *reinterpret_cast<const float4*>(kT + d * PF_ATT_PAD + 4 * kj);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int w = 0; w < 4; ++w) s[u][w] = __fmaf_rn(qa[u], ka[w], s[u][w]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < 4; ++w) s[u][w] = __fmul_rn(s[u][w], a.scale);
    };

    // ---- pass 1: row maxima ----
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (uint32_t k0 = 0; k0 < n_keys; k0 += PF_ATT_KC) {
        __syncthreads();
        load_k(k0);
        __syncthreads();
        float s[4][4];
        scores(s);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < 4; ++w)
                if (k0 + 4 * kj + w <= my_last[u]) m4[u] = fmaxf(m4[u], s[u][w]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) red[(4 * qi + u) * 16 + kj] = m4[u];
    __syncthreads();
    if (tid < PF_ATT_Q) {
        float m = -INFINITY;
        for (int i = 0; i < 16; ++i) m = fmaxf(m, red[tid * 16 + i]);
        rmax[tid] = m;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) m4[u] = rmax[4 * qi + u];

    // ---- pass 2: exponentials, sums, P.V ----
    const uint32_t ov = tid / 16, od = (tid % 16) * (HD / 16);  // output: vectors 4ov..+3, dims od..
    constexpr int DPT = HD / 16;                                // dims per thread (8 at hd 128)
    float acc[4][DPT];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[u][e] = 0.0f;
    float l4[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t k0 = 0; k0 < n_keys; k0 += PF_ATT_KC) {
        __syncthreads();
        load_k(k0);
        for (uint32_t i = tid; i < PF_ATT_KC * (HD / 4); i += PF_ATT_THREADS) {
            const uint32_t j = i / (HD / 4), c = i % (HD / 4);
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + j < n_keys) x = __ldg(reinterpret_cast<const float4*>(head + (size_t)(k0 + j) * 2 * HD + HD) + c);
            *reinterpret_cast<float4*>(vs + j * HD + 4 * c) = x;
        }
        __syncthreads();
        float s[4][4];
        scores(s);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint32_t key = k0 + 4 * kj + w;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float p = 0.0f;
                if (key <= my_last[u]) {
                    const float x = __fsub_rn(s[u][w], m4[u]);
                    p = key < nv ? exp_poly(x) : expf(x);
                }
                l4[u] = __fadd_rn(l4[u], p);
                pT[(4 * kj + w) * PF_ATT_PAD + 4 * qi + u] = p;
            }
        }
        __syncthreads();
#pragma unroll 4
        for (uint32_t j = 0; j < PF_ATT_KC; ++j) {
            const float4 pv = *reinterpret_cast<const float4*>(pT + j * PF_ATT_PAD + 4 * ov);
            const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
            float vv[DPT];
            if constexpr (DPT % 4 == 0) {
#pragma unroll
                for (int e = 0; e < DPT; e += 4) {
                    const float4 x = *reinterpret_cast<const float4*>(vs + j * HD + od + e);
                    vv[e] = x.x;
                    vv[e + 1] = x.y;
                    vv[e + 2] = x.z;
                    vv[e + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int e = 0; e < DPT; ++e) vv[e] = vs[j * HD + od + e];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int e = 0; e < DPT; ++e) acc[u][e] = __fmaf_rn(pa[u], vv[e], acc[u][e]);
        }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) red2[(4 * qi + u) * 16 + kj] = l4[u];
    __syncthreads();
    if (tid < PF_ATT_Q) {
        float l = 0.0f;
        for (int i = 0; i < 16; ++i) l += red2[tid * 16 + i];
        rinv[tid] = __fdiv_rn(1.0f, l);
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint32_t v = 4 * ov + u, row = r0 + v / G;
        if (row >= a.S) continue;
        const float inv = rinv[v];
        float* o = a.out + (size_t)row * D + (h * G + v % G) * HD + od;
#pragma unroll
        for (int e = 0; e < DPT; ++e) o[e] = __fmul_rn(acc[u][e], inv);
    }
}

// ---- causal attention of a prompt on the tensor cores ----------------------------------
// Same mathematics as attn_prefill_kernel (two passes: row maxima, then
// upstream's softmax and P.V), with the two products on mma.sync m16n8k16
// (f16 in, f32 accumulate), every operand as fp16 hi + lo halves after a
// power-of-two scale (per CTA for q, per 64-key chunk for K and for V, all
// multiplied back exactly) and three MMAs per product (hi*hi, hi*lo, lo*hi).
// Each chunk's P.V is summed in its own accumulators (12 MMAs) and added to
// the output in fp32, so the tensor core's truncating accumulation never
// runs long.  CTA = one KV head x 64 query vectors (its G query heads x 64/G
// rows); 4 warps, warp w owns vectors 16w..16w+15 (one m16 tile).
static constexpr uint32_t PT_Q = 64, PT_KC = 64, PT_THREADS = 128;
static constexpr uint32_t PT_LD = 136;  // padded row of the fp16 tiles (halves): conflict-free ldmatrix

__host__ __device__ inline size_t pf_attn_tc_smem(uint32_t hd) {
    // qh, ql [Q][LD] | kh, kl [KC][LD] | vh, vl [KC][LD] (fp16) | scales
    (void)hd;
    return ((size_t)PT_Q * PT_LD * 2 + (size_t)PT_KC * PT_LD * 4) * 2 + 64;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Block-wide max of |x| over the CTA (128 threads) -> the power-of-two
// exponent that maps it into [2^14, 2^15).
__device__ __forceinline__ int pt_block_exponent(float m, float* red) {
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    const float t = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    return pf_exponent(t);
}

template <int HD, int G>
__global__ void __launch_bounds__(PT_THREADS) attn_prefill_tc_kernel(const PfAttnArgs a) {
    static_assert(HD == 128, "tensor-core prompt attention: head_dim 128");
    static_assert(PT_Q % G == 0, "query vectors per CTA");
    constexpr uint32_t RQ = PT_Q / G;
    extern __shared__ __align__(16) uint8_t ptsm[];
    __half* qh = reinterpret_cast<__half*>(ptsm);
    __half* ql = qh + PT_Q * PT_LD;
    __half* kh = ql + PT_Q * PT_LD;
    __half* kl = kh + PT_KC * PT_LD;
    __half* vh = kl + PT_KC * PT_LD;
    __half* vl = vh + PT_KC * PT_LD;
    float* red = reinterpret_cast<float*>(vl + PT_KC * PT_LD);  // [4]
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t g = lane >> 2, t = lane & 3;
    const uint32_t h = blockIdx.y, r0 = blockIdx.x * RQ;
    const uint32_t D = a.n_heads * HD;
    const float* head = a.kv + (size_t)h * a.max_seq * 2 * HD;
    const uint32_t N = a.pos + a.S, nv = N / 8 * 8;
    const uint32_t last_row = min(a.S, r0 + RQ) - 1;
    const uint32_t n_keys = a.pos + last_row + 1;

    // ---- q: 64 vectors x 128, scaled, as hi / lo halves ----
    float qmax = 0.0f;
    for (uint32_t i = tid; i < PT_Q * (HD / 4); i += PT_THREADS) {
        const uint32_t v = i / (HD / 4), c = i % (HD / 4), row = r0 + v / G;
        if (row < a.S) {
            const float4 x = __ldg(reinterpret_cast<const float4*>(a.q + (size_t)row * D + (h * G + v % G) * HD) + c);
            qmax = fmaxf(qmax, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
    }
    const int eq = pt_block_exponent(qmax, red);
    const float qmul = ldexpf(1.0f, eq);
    for (uint32_t i = tid; i < PT_Q * (HD / 4); i += PT_THREADS) {
        const uint32_t v = i / (HD / 4), c = i % (HD / 4), row = r0 + v / G;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < a.S) x = __ldg(reinterpret_cast<const float4*>(a.q + (size_t)row * D + (h * G + v % G) * HD) + c);
        __half h0, l0, h1, l1, h2, l2, h3, l3;
        pf_split(x.x * qmul, h0, l0);
        pf_split(x.y * qmul, h1, l1);
        pf_split(x.z * qmul, h2, l2);
        pf_split(x.w * qmul, h3, l3);
        *reinterpret_cast<uint2*>(qh + v * PT_LD + 4 * c) = make_uint2(h2_bits(__halves2half2(h0, h1)), h2_bits(__halves2half2(h2, h3)));
        *reinterpret_cast<uint2*>(ql + v * PT_LD + 4 * c) = make_uint2(h2_bits(__halves2half2(l0, l1)), h2_bits(__halves2half2(l2, l3)));
    }
    // one K or V chunk (keys k0 .. k0+63, rows past n_keys zero) -> hi / lo
    // halves scaled by the chunk's power of two; returns 2^-e
    auto load_chunk = [&](uint32_t k0, uint32_t off, __half* dh, __half* dl) -> float {
        float m = 0.0f;
        for (uint32_t i = tid; i < PT_KC * (HD / 4); i += PT_THREADS) {
            const uint32_t j = i / (HD / 4), c = i % (HD / 4);
            if (k0 + j < n_keys) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(head + (size_t)(k0 + j) * 2 * HD + off) + c);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            }
        }
        const int e = pt_block_exponent(m, red);
        const float mul = ldexpf(1.0f, e);
        for (uint32_t i = tid; i < PT_KC * (HD / 4); i += PT_THREADS) {
            const uint32_t j = i / (HD / 4), c = i % (HD / 4);
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + j < n_keys) x = __ldg(reinterpret_cast<const float4*>(head + (size_t)(k0 + j) * 2 * HD + off) + c);
            __half h0, l0, h1, l1, h2, l2, h3, l3;
            pf_split(x.x * mul, h0, l0);
            pf_split(x.y * mul, h1, l1);
            pf_split(x.z * mul, h2, l2);
            pf_split(x.w * mul, h3, l3);
            *reinterpret_cast<uint2*>(dh + j * PT_LD + 4 * c) = make_uint2(h2_bits(__halves2half2(h0, h1)), h2_bits(__halves2half2(h2, h3)));
            *reinterpret_cast<uint2*>(dl + j * PT_LD + 4 * c) = make_uint2(h2_bits(__halves2half2(l0, l1)), h2_bits(__halves2half2(l2, l3)));
        }
        return ldexpf(1.0f, -e);
    };
    // S[8 key tiles][4] of this warp's 16 vectors against the chunk in kh/kl
    const uint32_t qa_h = smem_u32(qh) + ((16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1)) * PT_LD + 8 * (lane >> 4)) * 2;
    const uint32_t qa_l = qa_h + (uint32_t)((ql - qh) * 2);
    // B (keys x dims) for ldmatrix.x4: matrices (keys 0-7, dims 0-7 | 8-15) of tile n, and of tile n+1
    const uint32_t kb_h = smem_u32(kh) + (((lane & 7) + 8 * (lane >> 4)) * PT_LD + 8 * ((lane >> 3) & 1)) * 2;
    const uint32_t kb_l = kb_h + (uint32_t)((kl - kh) * 2);
    auto scores = [&](float (&S)[8][4]) {
#pragma unroll
        for (int n = 0; n < 8; ++n) S[n][0] = S[n][1] = S[n][2] = S[n][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            uint32_t ah[4], al[4];
            ldsm_x4(qa_h + ks * 32, ah[0], ah[1], ah[2], ah[3]);
            ldsm_x4(qa_l + ks * 32, al[0], al[1], al[2], al[3]);
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                uint32_t bh0, bh1, bh2, bh3, bl0, bl1, bl2, bl3;
                ldsm_x4(kb_h + (n * 8 * PT_LD + ks * 16) * 2, bh0, bh1, bh2, bh3);
                ldsm_x4(kb_l + (n * 8 * PT_LD + ks * 16) * 2, bl0, bl1, bl2, bl3);
                mma16816(S[n], ah, bh0, bh1);
                mma16816(S[n], ah, bl0, bl1);
                mma16816(S[n], al, bh0, bh1);
                mma16816(S[n + 1], ah, bh2, bh3);
                mma16816(S[n + 1], ah, bl2, bl3);
                mma16816(S[n + 1], al, bh2, bh3);
            }
        }
    };
    // this lane's rows: vectors 16 warp + g (e < 2) and + 8 (e >= 2)
    uint32_t last[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) last[hh] = a.pos + r0 + (16 * warp + g + 8 * hh) / G;
    const float unq = ldexpf(1.0f, -eq);

    // ---- pass 1: row maxima ----
    float mx[2] = {-INFINITY, -INFINITY};
    for (uint32_t k0 = 0; k0 < n_keys; k0 += PT_KC) {
        __syncthreads();
        const float unk = load_chunk(k0, 0, kh, kl);
        __syncthreads();
        float S[8][4];
        scores(S);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t key = k0 + 8 * n + 2 * t + (e & 1);
                const float sv = __fmul_rn(S[n][e] * unq * unk, a.scale);
                if (key <= last[e >> 1]) mx[e >> 1] = fmaxf(mx[e >> 1], sv);
            }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 1));
        mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 2));
    }

    // ---- pass 2: exponentials, sums, P.V ----
    float O[16][4];
#pragma unroll
    for (int d = 0; d < 16; ++d) O[d][0] = O[d][1] = O[d][2] = O[d][3] = 0.0f;
    float l[2] = {0.0f, 0.0f};
    // V (keys x dims) with .trans: matrices (keys 0-7 | 8-15) x (dims of tile d | d+1)
    const uint32_t vb_h = smem_u32(vh) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * PT_LD + 8 * (lane >> 4)) * 2;
    const uint32_t vb_l = vb_h + (uint32_t)((vl - vh) * 2);
    for (uint32_t k0 = 0; k0 < n_keys; k0 += PT_KC) {
        __syncthreads();
        const float unk = load_chunk(k0, 0, kh, kl);
        const float unv = load_chunk(k0, HD, vh, vl);
        __syncthreads();
        float S[8][4];
        scores(S);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t key = k0 + 8 * n + 2 * t + (e & 1);
                float p = 0.0f;
                if (key <= last[e >> 1]) {
                    const float x = __fsub_rn(__fmul_rn(S[n][e] * unq * unk, a.scale), mx[e >> 1]);
                    p = key < nv ? exp_poly(x) : expf(x);
                }
                l[e >> 1] = __fadd_rn(l[e >> 1], p);
                S[n][e] = p;
            }
        // P (C fragments) -> A fragments, hi and lo halves; this chunk's P.V
        float Oc[16][4];
#pragma unroll
        for (int d = 0; d < 16; ++d) Oc[d][0] = Oc[d][1] = Oc[d][2] = Oc[d][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < PT_KC / 16; ++ks) {
            uint32_t ph[4], pl[4];
            const float* s0 = S[2 * ks];
            const float* s1 = S[2 * ks + 1];
            const float src[4][2] = {{s0[0], s0[1]}, {s0[2], s0[3]}, {s1[0], s1[1]}, {s1[2], s1[3]}};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const __half2 hv = __floats2half2_rn(src[r][0], src[r][1]);
                const float2 hf = __half22float2(hv);
                ph[r] = h2_bits(hv);
                pl[r] = h2_bits(__floats2half2_rn(src[r][0] - hf.x, src[r][1] - hf.y));
            }
#pragma unroll
            for (int d = 0; d < 16; d += 2) {
                uint32_t bh0, bh1, bh2, bh3, bl0, bl1, bl2, bl3;
                ldsm_x4_t(vb_h + (ks * 16 * PT_LD + d * 8) * 2, bh0, bh1, bh2, bh3);
                ldsm_x4_t(vb_l + (ks * 16 * PT_LD + d * 8) * 2, bl0, bl1, bl2, bl3);
                mma16816(Oc[d], ph, bh0, bh1);
                mma16816(Oc[d], ph, bl0, bl1);
                mma16816(Oc[d], pl, bh0, bh1);
                mma16816(Oc[d + 1], ph, bh2, bh3);
                mma16816(Oc[d + 1], ph, bl2, bl3);
                mma16816(Oc[d + 1], pl, bh2, bh3);
            }
        }
#pragma unroll
        for (int d = 0; d < 16; ++d)
#pragma unroll
            for (int e = 0; e < 4; ++e) O[d][e] = __fadd_rn(O[d][e], Oc[d][e] * unv);
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        l[hh] += __shfl_xor_sync(0xffffffffu, l[hh], 1);
        l[hh] += __shfl_xor_sync(0xffffffffu, l[hh], 2);
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const uint32_t v = 16 * warp + g + 8 * hh, row = r0 + v / G;
        if (row >= a.S) continue;
        const float inv = __fdiv_rn(1.0f, l[hh]);
        float* o = a.out + (size_t)row * D + (h * G + v % G) * HD;
#pragma unroll
        for (int d = 0; d < 16; ++d)
            *reinterpret_cast<float2*>(o + 8 * d + 2 * t) =
                make_float2(__fmul_rn(O[d][2 * hh], inv), __fmul_rn(O[d][2 * hh + 1], inv));
    }
}

}  // namespace qb200
