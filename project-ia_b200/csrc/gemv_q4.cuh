// gemv_q4.cuh — Q4_0 dequant-GEMV for batch-1 decode (sm_100a).
//
// Replaces upstream q_gemv_q4_f32_avx2 (src/ops/avx2/matmul.c:98-271) and
// the elementwise kernels around it: the RMSNorm before a projection
// (src/ops/avx2/rmsnorm.c:15-92) runs as the prologue, and RoPE + KV-cache
// store (src/models/model.c:1170-1222, src/ops/avx2/rope.c:23-110), SiLU*up
// (silu.c:18-94 + mul_fp32.c:17-127) and the residual add (add_fp32.c:17-165)
// run as epilogues.
//
// Arithmetic.  A Q4_0 block contributes s * sum_k (q_k - 8) x_k.  The kernel
// evaluates sum_k q_k x_k EXACTLY on the integer tensor cores: the block's 32
// inputs are put on a common fixed-point grid (X_k = rint(x_k * 2^(22-e)),
// e the exponent of the block max, |X_k| < 2^22) and split into three signed
// int8 limbs (X = a*65536 + b*256 + c); one mma.sync m16n8k32 u8 x s8 -> s32
// multiplies 16 weight rows (q as u8, no float conversion at all) by the
// three limb columns with exact int32 sums.  The limbs are recombined and
// the -8*sum(X) term added in fp32, then scaled by s * 2^-(22-e).  The only
// approximations are the 2^-23 (relative to the block max) input grid and
// fp32 accumulation across blocks — the error of an fp32 dot product.
// Versus dequantising to fp32 this needs ~1.4 instead of ~4 instructions
// per weight, so the kernel is HBM-bound rather than issue-bound.
//
// Device weight layout ("slab tiles"): rows in slabs of 16; for each
// (slab, block) 320 bytes: 256 bytes of mma A fragments (lane-major, 8 bytes
// per lane: low nibbles = k 4t..4t+3, high nibbles = k 16+4t..16+4t+3 for
// rows g and g+8, g = lane/4, t = lane%4) then 16 fp32 scales laid out
// [g][row g, row g+8].  Blocks of a slab are contiguous, slabs follow each
// other, so any range of blocks is one 1-D bulk copy.
//
// Work split.  The grid's CTAs take equal contiguous ranges of the block
// sequence (slab-major), so every CTA streams the same bytes.  A slab cut
// by a range boundary is finished by the last of its CTAs to arrive
// (per-slab ticket in global scratch), which adds the parts in CTA order.
// Inside a CTA a producer warp streams stages through a shared-memory ring
// with cp.async.bulk + mbarrier; weight loads start before the programmatic
// dependent launch wait.  Consumer warp w handles the blocks of a slab with
// index = w (mod 8), so all sums run in a fixed order (deterministic).
#pragma once

#include "common.cuh"

namespace qb200 {

enum GemvEpilogue : int {
    EPI_STORE = 0,   // y[row] = v
    EPI_RESID = 1,   // y[row] = resid[row] + v  (resid may alias y)
    EPI_QKV = 2,     // rows [q | k | v]: RoPE q->y, RoPE k->cache, v->cache
    EPI_SILU = 3,    // rows interleaved (gate_i, up_i): y[i] = silu(gate_i) * up_i
};

struct StepParams {  // device-resident per-step scalars (graph-replay friendly)
    uint32_t token;  // current token id
    uint32_t pos;    // position of the current token
    uint32_t n_row;  // softmax row length (upstream N: pos+seq_len of the call)
    uint32_t valid;  // positions 0..valid-1 are unmasked for this row
};

static constexpr int GEMV_CONSUMER_WARPS = 8;
static constexpr int GEMV_THREADS = GEMV_CONSUMER_WARPS * 32 + 32;
static constexpr uint32_t GEMV_BLOCK_BYTES = 320;  // one (slab, block) unit
static constexpr uint32_t GEMV_BFRAG_BYTES = 96;   // x limb fragments of a block (12 lanes)
static constexpr int GEMV_XREGS = 8;               // input float4s per thread per batch
// An RMSNorm prologue needs the whole input in one register batch.
static constexpr uint32_t GEMV_MAX_NORM_K = GEMV_CONSUMER_WARPS * 32 * GEMV_XREGS * 4;

struct GemvArgs {
    const uint8_t* w;          // packed slab tiles
    uint32_t M, K;             // rows, cols
    uint32_t n_slabs, nb;      // slabs of 16 rows, blocks per row
    uint32_t stage_blocks;     // blocks per ring stage
    uint32_t n_stage;          // ring depth
    uint32_t max_parts;        // CTAs that can share one slab
    uint32_t red_slabs;        // slab sums a CTA holds in shared memory between reductions
    const float* x;            // input vector, or the embedding table if gather
    const StepParams* step;    // per-step scalars (token, pos)
    uint32_t gather;           // non-zero: x row = x + step->token * K (embedding)
    const float* norm_w;       // non-null: RMSNorm prologue with these gains
    float eps;
    float* x_copy;             // non-null: CTA 0 stores the raw input here
    float* y;
    const float* resid;
    int epi;
    float* part;               // scratch [n_slabs][max_parts][16]
    uint32_t* ticket;          // scratch [n_slabs], zero between launches
    // EPI_QKV
    const float* rope_cos;     // [max_seq][hd] duplicated-pair tables
    const float* rope_sin;
    float* kv_layer;           // [n_kv][max_seq][2*hd] of this layer
    uint32_t hd, q_rows, kv_rows, max_seq;
    unsigned long long* trace;  // step-trace slot (null: off)
};

// Shared memory: ring | bfrag[nb][96] | fsc[nb] float2 | red[red_slabs][8][16] | bars | misc
__host__ __device__ inline size_t gemv_smem_bytes(uint32_t nb, uint32_t stage_blocks,
                                                  uint32_t n_stage, uint32_t red_slabs) {
    return (size_t)n_stage * stage_blocks * GEMV_BLOCK_BYTES + (size_t)nb * GEMV_BFRAG_BYTES +
           (size_t)nb * 8 + (size_t)red_slabs * GEMV_CONSUMER_WARPS * 16 * 4 + 2 * 8 * 8 +
           64 * 4 + 128;
}

// CTA i owns blocks [n*i/G, n*(i+1)/G) of the slab-major block sequence
// (host guarantees n * G < 2^32, so 32-bit arithmetic is exact).
__host__ __device__ inline uint32_t range_begin(uint32_t n, uint32_t i, uint32_t G) {
    return n * i / G;
}

// Largest CTA index whose range starts at or before block x.
__device__ __forceinline__ uint32_t cta_of(uint32_t n, uint32_t G, uint32_t x) {
    uint32_t i = x * G / n;
    while (i + 1 < G && range_begin(n, i + 1, G) <= x) ++i;
    while (i > 0 && range_begin(n, i, G) > x) --i;
    return i;
}

__device__ __forceinline__ void rope_pair(float v0, float v1, const float* ct,
                                          const float* st, uint32_t e, float& o0,
                                          float& o1) {
    // upstream rope.c:79-96 (addsub of two unfused products)
    o0 = __fsub_rn(__fmul_rn(v0, ct[e]), __fmul_rn(v1, st[e]));
    o1 = __fadd_rn(__fmul_rn(v1, ct[e + 1]), __fmul_rn(v0, st[e + 1]));
}

__device__ __forceinline__ void mma_u8s8(int d[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Epilogue for lanes 0..15 of one warp holding the 16 finished rows of slab j
// (lane = row within the slab).  Pairs use the odd lane's value via shuffle.
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, uint32_t j, uint32_t lane, float v) {
    const float vn = __shfl_down_sync(0x0000ffffu, v, 1, 16);
    const uint32_t row = j * 16 + lane;
    if (row >= a.M) return;
    if (a.epi == EPI_STORE) {
        a.y[row] = v;
    } else if (a.epi == EPI_RESID) {
        a.y[row] = __fadd_rn(a.resid[row], v);
    } else if (lane & 1) {
        return;  // pairs: the even lane writes both
    } else if (a.epi == EPI_SILU) {
        // upstream silu.c (poly exp on the vector body) then mul_fp32.c
        a.y[row / 2] = __fmul_rn(silu_poly(v), vn);
    } else {  // EPI_QKV
        const uint32_t pos = a.step->pos;
        const float* ct = a.rope_cos + (size_t)pos * a.hd;
        const float* st = a.rope_sin + (size_t)pos * a.hd;
        float o0, o1;
        if (row < a.q_rows) {
            rope_pair(v, vn, ct, st, row % a.hd, o0, o1);
            a.y[row] = o0;
            a.y[row + 1] = o1;
        } else if (row < a.q_rows + a.kv_rows) {
            const uint32_t kr = row - a.q_rows, h = kr / a.hd, e = kr % a.hd;
            rope_pair(v, vn, ct, st, e, o0, o1);
            float* dst = a.kv_layer + ((size_t)h * a.max_seq + pos) * 2 * a.hd + e;
            dst[0] = o0;
            dst[1] = o1;
        } else {
            const uint32_t vr = row - a.q_rows - a.kv_rows, h = vr / a.hd, e = vr % a.hd;
            float* dst = a.kv_layer + ((size_t)h * a.max_seq + pos) * 2 * a.hd + a.hd + e;
            dst[0] = v;
            dst[1] = vn;
        }
    }
}

#ifdef QB200_GEMV_PHASES  // experiment builds only: per-CTA phase timestamps
__device__ unsigned long long g_gemv_phase[2048 * 8];
#define GEMV_PHASE(i, v) (g_gemv_phase[blockIdx.x * 8 + (i)] = (v))
#else
#define GEMV_PHASE(i, v) ((void)0)
#endif

__global__ void __launch_bounds__(GEMV_THREADS, 2) gemv_q4_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t NW = GEMV_CONSUMER_WARPS, T = NW * 32;
    const uint32_t nb = a.nb;
    const uint32_t stage_bytes = a.stage_blocks * GEMV_BLOCK_BYTES;
    uint8_t* ring = smem;
    uint8_t* bfrag = ring + (size_t)a.n_stage * stage_bytes;
    float2* fsc = reinterpret_cast<float2*>(bfrag + (size_t)nb * GEMV_BFRAG_BYTES);
    float* red = reinterpret_cast<float*>(fsc + nb);             // [red_slabs][NW][16]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)a.red_slabs * NW * 16);
    uint64_t* empty = full + 8;
    float* rms_part = reinterpret_cast<float*>(empty + 8);   // [NW]

    const uint32_t tid = threadIdx.x;
    const uint32_t G = gridDim.x, cta = blockIdx.x;
    const uint32_t NB = a.n_slabs * nb;
    const uint32_t x0 = range_begin(NB, cta, G), x1 = range_begin(NB, cta + 1, G);
    // Only the first and last slab of the range can be shared with other
    // CTAs; resolve their owners once, here.
    const uint32_t j_first = x0 / nb, j_last = (x1 - 1) / nb;
    uint32_t own_lo[2] = {cta, cta}, own_hi[2] = {cta, cta};  // [first slab, last slab]
    if (j_first * nb < x0 || (j_first + 1) * nb > x1) {
        own_lo[0] = cta_of(NB, G, j_first * nb);
        own_hi[0] = cta_of(NB, G, j_first * nb + nb - 1);
    }
    if (j_last != j_first && (j_last + 1) * nb > x1) {
        own_lo[1] = cta;
        own_hi[1] = cta_of(NB, G, j_last * nb + nb - 1);
    }
    const uint32_t n_stages = (x1 - x0 + a.stage_blocks - 1) / a.stage_blocks;

    if (tid == 0) {
        for (uint32_t s = 0; s < a.n_stage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) trace_mark(a.trace, 0);
    if (tid == 0) GEMV_PHASE(0, gtimer());
    pdl_trigger();

    if (tid >= T) {
        // ---- producer warp: stream this CTA's block range -------------------
        if (tid == T) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t s = 0, ph = 0;  // ring slot and its phase parity
            for (uint32_t k = 0, b0 = x0; k < n_stages; ++k, b0 += a.stage_blocks) {
                if (k >= a.n_stage && !mbar_wait(&empty[s], ph ^ 1, QDEV_WAIT_EMPTY_TIMEOUT)) break;
                const uint32_t n = min(a.stage_blocks, x1 - b0);
                mbar_arrive_expect_tx(&full[s], n * GEMV_BLOCK_BYTES);
                bulk_g2s(ring + (size_t)s * stage_bytes, a.w + (size_t)b0 * GEMV_BLOCK_BYTES,
                         n * GEMV_BLOCK_BYTES, &full[s], pol);
                if (++s == a.n_stage) {
                    s = 0;
                    ph ^= 1;
                }
            }
            GEMV_PHASE(5, gtimer());
        }
        pdl_wait();  // every thread waits: the grid ends after its predecessor
        return;
    }

    // ---- consumers: input prologue -------------------------------------------
    pdl_wait();
    if (tid == 0) trace_mark(a.trace, 1);
    if (tid == 0) GEMV_PHASE(1, gtimer());
    const uint32_t lane = tid & 31, warp = tid >> 5;
    const float* xs = a.x;
    if (a.gather) xs = a.x + (size_t)a.step->token * a.K;
    // All input loads are issued at once (float4, registers); a serial loop
    // of dependent L2 loads here would delay the whole stream by microseconds.
    // Thread tid holds float4 number tid + T*r; 8 consecutive threads hold
    // one 32-element Q4 block.
    constexpr int NR = GEMV_XREGS;
    const uint32_t n4 = a.K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    const float4* g4 = reinterpret_cast<const float4*>(a.norm_w);
    float r_norm = 1.0f;
    for (uint32_t base = 0; base < n4; base += T * NR) {
        float4 xv[NR], gv[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const uint32_t i = base + tid + T * r;
            xv[r] = i < n4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            gv[r] = (g4 && i < n4) ? g4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (a.x_copy && cta == 0) {
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint32_t i = base + tid + T * r;
                if (i < n4) reinterpret_cast<float4*>(a.x_copy)[i] = xv[r];
            }
        }
        if (a.norm_w && base == 0) {
            // upstream rmsnorm.c: mean of squares, rsqrt + one Newton step
            // (the host only pairs a norm with K <= T*NR*4, one batch)
            float ss = 0.0f;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                ss = __fmaf_rn(xv[r].x, xv[r].x, ss);
                ss = __fmaf_rn(xv[r].y, xv[r].y, ss);
                ss = __fmaf_rn(xv[r].z, xv[r].z, ss);
                ss = __fmaf_rn(xv[r].w, xv[r].w, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) rms_part[warp] = ss;
            asm volatile("bar.sync 1, %0;" ::"r"(T));
            float tot = 0.0f;
            for (uint32_t i = 0; i < NW; ++i) tot += rms_part[i];
            float me = __fadd_rn(__fdiv_rn(tot, (float)a.K), a.eps);
            float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
            float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
            r_norm = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
        }
        // Fixed-point limbs: B fragment of lane L = g*4 + t (g < 3 = limb):
        // word 0 = limb g of k 4t..4t+3, word 1 = limb g of k 16+4t..16+4t+3.
        // This thread's float4 is k = 4*sub..4*sub+3 of its block, i.e.
        // t = sub % 4, word = sub / 4: one 32-bit store per limb.
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const uint32_t i = base + tid + T * r;
            if (base + T * r >= n4) break;  // uniform: whole warp past the end
            float4 v = xv[r];
            if (a.norm_w) {
                v.x = __fmul_rn(__fmul_rn(v.x, r_norm), gv[r].x);
                v.y = __fmul_rn(__fmul_rn(v.y, r_norm), gv[r].y);
                v.z = __fmul_rn(__fmul_rn(v.z, r_norm), gv[r].z);
                v.w = __fmul_rn(__fmul_rn(v.w, r_norm), gv[r].w);
            }
            float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            // Grid 2^-sh with sh = 22 - e, m = f 2^e (f in [0.5, 1)): for a
            // normal m, e = E - 126 with E its biased exponent field.  A
            // subnormal m uses E = 1 (a coarser grid, still |X| <= 2^22), an
            // all-zero block any E.  v 2^sh is formed as two exact
            // power-of-two products (sh spans -106..147); an intermediate
            // can only lose bits when the final value rounds to 0 anyway.
            const int E = m > 0.0f ? max((int)(__float_as_uint(m) >> 23), 1) : 126;
            const int sh = 148 - E, s1 = sh >> 1, s2 = sh - s1;
            const float p1 = __int_as_float((s1 + 127) << 23), p2 = __int_as_float((s2 + 127) << 23);
            const int X[4] = {__float2int_rn(__fmul_rn(__fmul_rn(v.x, p1), p2)),
                              __float2int_rn(__fmul_rn(__fmul_rn(v.y, p1), p2)),
                              __float2int_rn(__fmul_rn(__fmul_rn(v.z, p1), p2)),
                              __float2int_rn(__fmul_rn(__fmul_rn(v.w, p1), p2))};
            uint32_t la = 0, lb = 0, lc = 0;
            int sx = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int c8 = (int)(int8_t)(X[q] & 0xFF);
                const int X1 = (X[q] - c8) >> 8;
                const int b8 = (int)(int8_t)(X1 & 0xFF);
                const int a8 = (X1 - b8) >> 8;
                la |= (uint32_t)(a8 & 0xFF) << (8 * q);
                lb |= (uint32_t)(b8 & 0xFF) << (8 * q);
                lc |= (uint32_t)(c8 & 0xFF) << (8 * q);
                sx += X[q];
            }
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
            if (i < n4) {
                const uint32_t b = i / 8, sub = i % 8;
                uint32_t* bf = reinterpret_cast<uint32_t*>(bfrag + (size_t)b * GEMV_BFRAG_BYTES);
                const uint32_t w = (sub % 4) * 2 + sub / 4;  // 32-bit word within a limb's 32 B
                bf[0 * 8 + w] = la;
                bf[1 * 8 + w] = lb;
                bf[2 * 8 + w] = lc;
                if (sub == 0) {
                    // 2^-sh = 2^(E-148): normal for E >= 22, else the
                    // subnormal 2^(E+1) * 2^-149
                    const float f = __uint_as_float(E >= 22 ? (uint32_t)(E - 21) << 23
                                                            : 1u << (E + 1));
                    fsc[b] = make_float2(f, f * (-8.0f * (float)sx));
                }
            }
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(T));
    if (tid == 0) GEMV_PHASE(2, gtimer());
#ifdef QB200_GEMV_PHASES
    unsigned long long ph_wait = 0, ph_flush = 0;
#endif

    // ---- main loop ---------------------------------------------------------------
    const uint32_t g = lane >> 2, t = lane & 3;
    // D fragment of lane (g, t): rows g and g+8, columns 2t, 2t+1.  Columns
    // 0..2 are the limbs (a, b, c); lanes t >= 2 and column 3 see whatever
    // B lanes 12..31 load (their rows of the limb table, reused) and are
    // cancelled by zero weights.  t = 0: p = 256*D_a + D_b, weight 256 f;
    // t = 1: p = D_c, weight f, plus the -8*sum(X) correction.
    const int m0 = t == 0 ? 256 : 1;
    const int m1 = t == 0 ? 1 : 0;
    const float wt = t == 0 ? 256.0f : (t == 1 ? 1.0f : 0.0f);
    const float ct = t == 1 ? 1.0f : 0.0f;
    const uint32_t ring_off = 0;
    const uint32_t bfrag_off = (uint32_t)(bfrag - smem) + (lane % 12) * 8;
    const uint32_t fsc_off = (uint32_t)(reinterpret_cast<uint8_t*>(fsc) - smem);
    // One block: bytes at smem + q (weights, lane part), + sq (scales of
    // rows g, g+8), + bq (limb fragment), + fq (grid factor, correction).
    auto block_terms = [&](uint32_t q_off, uint32_t b_off, uint32_t f_off, float& u0, float& u1,
                           float2& sc) {
        const uint2 q = *reinterpret_cast<const uint2*>(smem + q_off);
        sc = *reinterpret_cast<const float2*>(smem + q_off + (256 + g * 8 - lane * 8));
        const uint2 bv = *reinterpret_cast<const uint2*>(smem + b_off);
        const float2 fz = *reinterpret_cast<const float2*>(smem + f_off);
        int d[4];
#ifdef QB200_GEMV_NO_MMA  // experiment builds only
        d[0] = q.x ^ bv.x; d[1] = q.y ^ bv.y; d[2] = (q.x >> 4) ^ bv.y; d[3] = (q.y >> 4) ^ bv.x;
#else
        mma_u8s8(d, q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, (q.x >> 4) & 0x0F0F0F0Fu,
                 (q.y >> 4) & 0x0F0F0F0Fu, bv.x, bv.y);
#endif
        const float fw = fz.x * wt;
        const float fc = fz.y * ct;
        u0 = __fmaf_rn((float)(d[0] * m0 + d[1] * m1), fw, fc);
        u1 = __fmaf_rn((float)(d[2] * m0 + d[3] * m1), fw, fc);
    };
    // Slab sums wait in red[] (per warp) and are reduced by the whole CTA
    // every red_slabs slabs and at the end: warp w finishes slabs w, w+NW, ...
    // of the batch (cross-CTA parts through the ticket, then the epilogue).
    const uint32_t RS = a.red_slabs;
    uint32_t jl = 0, j_batch = j_first;
    auto reduce_batch = [&](uint32_t cnt) {
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        for (uint32_t r = warp; r < cnt; r += NW) {
            const uint32_t j = j_batch + r;
            float v = 0.0f;
            if (lane < 16)
#pragma unroll
                for (uint32_t w = 0; w < NW; ++w) v += red[(r * NW + w) * 16 + lane];
            const uint32_t c_first = j == j_first ? own_lo[0] : (j == j_last ? own_lo[1] : cta);
            const uint32_t c_last = j == j_first ? own_hi[0] : (j == j_last ? own_hi[1] : cta);
            bool finish = c_first == c_last;
            if (!finish) {
                float* pp = a.part + ((size_t)j * a.max_parts) * 16;
                if (lane < 16) pp[(cta - c_first) * 16 + lane] = v;
                __threadfence();
                uint32_t last = 0;
                if (lane == 0) last = atomicAdd(&a.ticket[j], 1u) == c_last - c_first ? 1u : 0u;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    v = 0.0f;
                    if (lane < 16)
                        for (uint32_t p = 0; p <= c_last - c_first; ++p) v += __ldcg(&pp[p * 16 + lane]);
                    if (lane == 0) a.ticket[j] = 0u;
                    finish = true;
                }
            }
            if (finish && lane < 16) gemv_epilogue(a, j, lane, v);
        }
        j_batch += cnt;
        jl = 0;
    };
    float acc0 = 0.0f, acc1 = 0.0f;
    // running ring slot / parity and current slab (no divisions per stage)
    uint32_t s = 0, ph = 0, j = j_first, jb = j_first * nb;
    for (uint32_t k = 0, sb0 = x0; k < n_stages; ++k, sb0 += a.stage_blocks) {
#ifdef QB200_GEMV_PHASES
        const unsigned long long pw0 = gtimer();
#endif
        mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
#ifdef QB200_GEMV_PHASES
        ph_wait += gtimer() - pw0;
        if (k == 0 && tid == 0) GEMV_PHASE(3, gtimer());
#endif
        const uint32_t sb1 = min(sb0 + a.stage_blocks, x1);
        for (uint32_t seg = sb0; seg < sb1;) {
            const uint32_t seg_end = min(sb1, jb + nb);
            // this warp's blocks of the segment: (b - jb) % NW == warp
            const uint32_t b = seg + ((warp + NW - (seg - jb) % NW) % NW);
            int n = b < seg_end ? (int)((seg_end - b + NW - 1) / NW) : 0;
#ifdef QB200_GEMV_NO_COMPUTE  // experiment builds only: stream without arithmetic
            n = 0;
#endif
            uint32_t qo = ring_off + s * stage_bytes + (b - sb0) * GEMV_BLOCK_BYTES + lane * 8;
            uint32_t bo = bfrag_off + (b - jb) * GEMV_BFRAG_BYTES;
            uint32_t fo = fsc_off + (b - jb) * 8;
            constexpr uint32_t QS = NW * GEMV_BLOCK_BYTES, BS = NW * GEMV_BFRAG_BYTES, FS = NW * 8;
            // four independent blocks per step, accumulated in block order
            for (; n >= 4; n -= 4, qo += 4 * QS, bo += 4 * BS, fo += 4 * FS) {
                float u[4][2];
                float2 sc[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    block_terms(qo + i * QS, bo + i * BS, fo + i * FS, u[i][0], u[i][1], sc[i]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc0 = __fmaf_rn(sc[i].x, u[i][0], acc0);
                    acc1 = __fmaf_rn(sc[i].y, u[i][1], acc1);
                }
            }
            for (; n > 0; --n, qo += QS, bo += BS, fo += FS) {
                float u0, u1;
                float2 sc;
                block_terms(qo, bo, fo, u0, u1, sc);
                acc0 = __fmaf_rn(sc.x, u0, acc0);
                acc1 = __fmaf_rn(sc.y, u1, acc1);
            }
            if (seg_end == jb + nb || seg_end == x1) {
#ifdef QB200_GEMV_PHASES
                const unsigned long long pf0 = gtimer();
#endif
                // slab j done for this warp: limbs (quad) -> red[jl][warp]
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
                if (t == 0) {
                    red[(jl * NW + warp) * 16 + g] = acc0;
                    red[(jl * NW + warp) * 16 + g + 8] = acc1;
                }
                acc0 = acc1 = 0.0f;
                if (++jl == RS) {
                    reduce_batch(RS);
                    asm volatile("bar.sync 1, %0;" ::"r"(T));  // red[] free again
                }
#ifdef QB200_GEMV_PHASES
                ph_flush += gtimer() - pf0;
#endif
            }
            if (seg_end == jb + nb) {
                ++j;
                jb += nb;
            }
            seg = seg_end;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == a.n_stage) {
            s = 0;
            ph ^= 1;
        }
    }
    if (jl) reduce_batch(jl);
    if (tid == 0) trace_mark(a.trace, 2);
#ifdef QB200_GEMV_PHASES
    if (tid == 0) {
        GEMV_PHASE(4, gtimer());
        GEMV_PHASE(6, ph_wait);
        GEMV_PHASE(7, ph_flush);
    }
#endif
}

// Repack upstream AoS Q4_0 blocks ([M][nb] x 20 B) into slab tiles.
// interleave_half != 0: destination row 2i takes source row i and 2i+1 takes
// source row interleave_half + i (gate/up pairing).  Rows >= M are zero.
__global__ void q4_pack_kernel(const uint8_t* __restrict__ src, uint32_t M, uint32_t K,
                               uint32_t interleave_half, uint8_t* __restrict__ dst) {
    const uint32_t nb = K / 32;
    const uint32_t n_slabs = (M + 15) / 16;
    const uint64_t n = (uint64_t)n_slabs * nb * 32;  // one thread per (slab, block, lane)
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t lane = (uint32_t)(i % 32);
        const uint64_t sb = i / 32;
        const uint32_t b = (uint32_t)(sb % nb), j = (uint32_t)(sb / nb);
        const uint32_t g = lane >> 2, t = lane & 3;
        uint8_t* out = dst + sb * GEMV_BLOCK_BYTES;
        uint32_t words[2];
        float scales[2];
        for (int half = 0; half < 2; ++half) {
            const uint32_t drow = j * 16 + g + 8 * half;
            uint32_t wv = 0;
            float sv = 0.0f;
            if (drow < M) {
                uint32_t srow = drow;
                if (interleave_half) srow = (drow & 1) ? interleave_half + drow / 2 : drow / 2;
                const uint8_t* blk = src + ((size_t)srow * nb + b) * 20;
                for (int by = 0; by < 4; ++by) {
                    const uint32_t klo = 4 * t + by, khi = 16 + 4 * t + by;
                    const uint32_t nlo = (blk[klo / 2] >> ((klo & 1) * 4)) & 15;
                    const uint32_t nhi = (blk[khi / 2] >> ((khi & 1) * 4)) & 15;
                    wv |= (nlo | (nhi << 4)) << (8 * by);
                }
                memcpy(&sv, blk + 16, 4);
            }
            words[half] = wv;
            scales[half] = sv;
        }
        *reinterpret_cast<uint2*>(out + lane * 8) = make_uint2(words[0], words[1]);
        if (t == 0) *reinterpret_cast<float2*>(out + 256 + g * 8) = make_float2(scales[0], scales[1]);
    }
}

}  // namespace qb200
