// gemv_q4.cuh — Q4_0 dequant-GEMV for batch-1 decode (sm_100a).
//
// Replaces upstream q_gemv_q4_f32_avx2 (src/ops/avx2/matmul.c:98-271) and
// the elementwise kernels around it: the RMSNorm before a projection
// (src/ops/avx2/rmsnorm.c:15-92) runs as the prologue, and RoPE + KV-cache
// store (src/models/model.c:1170-1222, src/ops/avx2/rope.c:23-110), SiLU*up
// (silu.c:18-94 + mul_fp32.c:17-127) and the residual add (add_fp32.c:17-165)
// run as epilogues.
//
// Device weight layout ("stream tiles"): rows are grouped R at a time; a
// tile is the R rows' 16-byte nibble planes ([R][nb][16], the upstream qs
// bytes unchanged) followed by their fp32 scales ([R][nb]), nb = K/32.
// Tiles are contiguous in HBM, so a tile is one 1-D bulk copy.
//
// CTA = (nb/BPT)*c consumer threads + 1 producer warp.  Consumer thread t
// owns the BPT block columns cb, cb+nb/BPT, ... (cb = t % (nb/BPT)) of every
// row r with r % c == t / (nb/BPT); its 32*BPT inputs live in registers for
// the whole kernel.  The producer warp streams this CTA's tiles through an
// NSTAGE shared-memory ring with cp.async.bulk + mbarrier (transaction
// bytes); weight loads do not depend on the previous kernel, so they start
// before the programmatic-dependent-launch wait.  Dequantisation builds
// 2^23+q floats with one PRMT per nibble, subtracts 2^23+8 exactly (packed
// FADD2) and accumulates with packed FFMA2; per row the block partials
// s_b*dot_b are summed by one warp from shared memory.
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

struct GemvArgs {
    const uint8_t* w;          // packed stream tiles
    uint32_t M, K, R, c;       // rows, cols, rows per tile, row groups per tile
    uint32_t bpt;              // Q4 blocks per consumer thread per row (template)
    uint32_t n_tiles;
    const float* x;            // input vector, or the embedding table if gather
    const StepParams* step;    // per-step scalars (token, pos)
    uint32_t gather;           // non-zero: x row = x + step->token * K (embedding)
    const float* norm_w;       // non-null: RMSNorm prologue with these gains
    float eps;
    float* x_copy;             // non-null: CTA 0 stores the raw input here
    float* y;
    const float* resid;
    int epi;
    // EPI_QKV
    const float* rope_cos;     // [max_seq][hd] duplicated-pair tables
    const float* rope_sin;
    float* kv_layer;           // [n_kv][max_seq][2*hd] of this layer
    uint32_t hd, q_rows, kv_rows, max_seq;
};

static constexpr int GEMV_NSTAGE = 4;
static constexpr int GEMV_MAX_CONSUMERS = 256;

__host__ __device__ inline uint32_t gemv_tile_bytes(uint32_t R, uint32_t K) {
    return R * (K / 32) * 20u;
}

// Shared memory: ring | red[2][R*nb/BPT] | barriers | rms partials
__host__ __device__ inline size_t gemv_smem_bytes(uint32_t R, uint32_t K, uint32_t bpt) {
    size_t tile = gemv_tile_bytes(R, K);
    size_t red = 2ull * R * (K / 32 / bpt) * 4;
    return GEMV_NSTAGE * tile + red + 2 * GEMV_NSTAGE * 8 + 64 * 4 + 64;
}

__device__ __forceinline__ void rope_pair(float v0, float v1, const float* ct,
                                          const float* st, uint32_t e, float& o0,
                                          float& o1) {
    // upstream rope.c:79-96 (addsub of two unfused products)
    o0 = __fsub_rn(__fmul_rn(v0, ct[e]), __fmul_rn(v1, st[e]));
    o1 = __fadd_rn(__fmul_rn(v1, ct[e + 1]), __fmul_rn(v0, st[e + 1]));
}

// BPT: Q4 blocks per thread per row; ROWS: rows per thread per tile (R / c).
template <int BPT, int ROWS>
__global__ void __launch_bounds__(GEMV_MAX_CONSUMERS + 32, 2) gemv_q4_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nb = a.K / 32;
    const uint32_t nbc = nb / BPT;       // block columns per row group
    const uint32_t T = nbc * a.c;        // consumer threads
    const uint32_t tile_bytes = gemv_tile_bytes(a.R, a.K);
    uint8_t* ring = smem;
    float* red = reinterpret_cast<float*>(smem + GEMV_NSTAGE * tile_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * a.R * nbc);
    uint64_t* empty = full + GEMV_NSTAGE;
    float* rms_part = reinterpret_cast<float*>(empty + GEMV_NSTAGE);

    const uint32_t tid = threadIdx.x;
    const uint32_t G = gridDim.x;
    const uint32_t t0 = (uint32_t)((uint64_t)a.n_tiles * blockIdx.x / G);
    const uint32_t t1 = (uint32_t)((uint64_t)a.n_tiles * (blockIdx.x + 1) / G);
    const uint32_t n_my = t1 - t0;
    const uint32_t n_cwarps = T / 32;

    if (tid == 0) {
        for (int s = 0; s < GEMV_NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], n_cwarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (tid >= T) {
        // ---- producer warp: stream this CTA's tiles ----------------------
        if (tid == T) {
            const uint64_t pol = l2_evict_first_policy();
            for (uint32_t k = 0; k < n_my; ++k) {
                const uint32_t s = k % GEMV_NSTAGE;
                if (k >= GEMV_NSTAGE &&
                    !mbar_wait(&empty[s], ((k / GEMV_NSTAGE) & 1) ^ 1, QDEV_WAIT_EMPTY_TIMEOUT))
                    break;
                mbar_arrive_expect_tx(&full[s], tile_bytes);
                bulk_g2s(ring + (size_t)s * tile_bytes,
                         a.w + (size_t)(t0 + k) * tile_bytes, tile_bytes, &full[s], pol);
            }
        }
        pdl_wait();  // every thread waits: the grid ends after its predecessor
        return;
    }

    // ---- consumers -----------------------------------------------------------
    pdl_wait();
    const uint32_t cb = tid % nbc, g = tid / nbc;
    const uint32_t lane = tid & 31, warp = tid >> 5;
    const float* xs = a.x;
    if (a.gather) xs = a.x + (size_t)a.step->token * a.K;

    float r_norm = 1.0f;
    if (a.norm_w) {
        // upstream rmsnorm.c: mean of squares, rsqrt + one Newton step
        float ss = 0.0f;
        for (uint32_t i = tid; i < a.K; i += T) ss = __fmaf_rn(xs[i], xs[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) rms_part[warp] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        float tot = 0.0f;
        for (uint32_t i = 0; i < n_cwarps; ++i) tot += rms_part[i];
        float me = __fadd_rn(__fdiv_rn(tot, (float)a.K), a.eps);
        float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
        float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
        r_norm = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
    }
    if (a.x_copy && blockIdx.x == 0)
        for (uint32_t i = tid; i < a.K; i += T) a.x_copy[i] = xs[i];

    float2 xr[BPT][16];
#pragma unroll
    for (int bi = 0; bi < BPT; ++bi) {
        const uint32_t b = cb + bi * nbc;
        const float4* x4 = reinterpret_cast<const float4*>(xs + (size_t)b * 32);
        const float4* g4 = a.norm_w ? reinterpret_cast<const float4*>(a.norm_w + (size_t)b * 32)
                                    : nullptr;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 v = x4[i];
            if (g4) {
                float4 gw = g4[i];
                v.x = __fmul_rn(__fmul_rn(v.x, r_norm), gw.x);
                v.y = __fmul_rn(__fmul_rn(v.y, r_norm), gw.y);
                v.z = __fmul_rn(__fmul_rn(v.z, r_norm), gw.z);
                v.w = __fmul_rn(__fmul_rn(v.w, r_norm), gw.w);
            }
            xr[bi][2 * i] = make_float2(v.x, v.y);
            xr[bi][2 * i + 1] = make_float2(v.z, v.w);
        }
    }

    const bool pairs = (a.epi == EPI_QKV || a.epi == EPI_SILU);
    const uint32_t units = pairs ? a.R / 2 : a.R;

    // Dequantisation: one PRMT moves a nibble (pre-masked into the low half
    // of a byte) under the exponent byte 0x4B, giving the float 2^23 + q; a
    // packed subtract of 2^23 + 8 then yields q - 8 exactly.  (Folding the
    // -8 into a block-sum correction instead saves that subtract but costs
    // ~4 bits through cancellation, which long-context attention amplified
    // past the parity tolerance.)
    const float2 bias = make_float2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
    for (uint32_t k = 0; k < n_my; ++k) {
        const uint32_t s = k % GEMV_NSTAGE;
        const bool ok = mbar_wait(&full[s], (k / GEMV_NSTAGE) & 1, QDEV_WAIT_FULL_TIMEOUT);
        const uint8_t* tile = ring + (size_t)s * tile_bytes;
        const uint4* qs = reinterpret_cast<const uint4*>(tile);
        const float* sc = reinterpret_cast<const float*>(tile + (size_t)a.R * nb * 16);
        float* rb = red + (k & 1) * a.R * nbc;
#pragma unroll
        for (int j = 0; j < ROWS; ++j) {
            const uint32_t r = g + a.c * j;
            float part = 0.0f;
#pragma unroll
            for (int bi = 0; bi < BPT; ++bi) {
                const uint32_t b = cb + bi * nbc;
                const uint4 q = qs[r * nb + b];
                const float scale = sc[r * nb + b];
                float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
                const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint32_t lo = words[wi] & 0x0F0F0F0Fu;
                    const uint32_t hi = (words[wi] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const uint32_t sel = 0x7540u | (uint32_t)m;
                        float2 d = make_float2(__uint_as_float(prmt(lo, 0x4B000000u, sel)),
                                               __uint_as_float(prmt(hi, 0x4B000000u, sel)));
                        d = __fadd2_rn(d, bias);  // exactly q - 8
                        if (m & 1) acc1 = __ffma2_rn(d, xr[bi][4 * wi + m], acc1);
                        else acc0 = __ffma2_rn(d, xr[bi][4 * wi + m], acc0);
                    }
                }
                const float dot =
                    __fadd_rn(__fadd_rn(acc0.x, acc0.y), __fadd_rn(acc1.x, acc1.y));
                part = __fmaf_rn(scale, dot, part);
            }
            rb[r * nbc + cb] = ok ? part : 0.0f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        asm volatile("bar.sync 1, %0;" ::"r"(T));

        // ---- per-row reduction + epilogue (one warp per row / row pair) ----
        const uint32_t tile_row0 = (t0 + k) * a.R;
        for (uint32_t u = warp; u < units; u += n_cwarps) {
            const uint32_t r0 = pairs ? 2 * u : u;
            float v0 = 0.0f, v1 = 0.0f;
            for (uint32_t i = lane; i < nbc; i += 32) {
                v0 += rb[r0 * nbc + i];
                if (pairs) v1 += rb[(r0 + 1) * nbc + i];
            }
            v0 = warp_sum(v0);
            if (pairs) v1 = warp_sum(v1);
            if (lane != 0) continue;
            const uint32_t row = tile_row0 + r0;
            if (row >= a.M) continue;
            if (a.epi == EPI_STORE) {
                a.y[row] = v0;
            } else if (a.epi == EPI_RESID) {
                a.y[row] = __fadd_rn(a.resid[row], v0);
            } else if (a.epi == EPI_SILU) {
                // upstream silu.c (poly exp on the vector body) then mul_fp32.c
                a.y[row / 2] = __fmul_rn(silu_poly(v0), v1);
            } else {  // EPI_QKV
                const uint32_t pos = a.step->pos;
                const float* ct = a.rope_cos + (size_t)pos * a.hd;
                const float* st = a.rope_sin + (size_t)pos * a.hd;
                float o0, o1;
                if (row < a.q_rows) {
                    rope_pair(v0, v1, ct, st, row % a.hd, o0, o1);
                    a.y[row] = o0;
                    a.y[row + 1] = o1;
                } else if (row < a.q_rows + a.kv_rows) {
                    const uint32_t kr = row - a.q_rows, h = kr / a.hd, e = kr % a.hd;
                    rope_pair(v0, v1, ct, st, e, o0, o1);
                    float* dst = a.kv_layer + ((size_t)h * a.max_seq + pos) * 2 * a.hd + e;
                    dst[0] = o0;
                    dst[1] = o1;
                } else {
                    const uint32_t vr = row - a.q_rows - a.kv_rows, h = vr / a.hd, e = vr % a.hd;
                    float* dst =
                        a.kv_layer + ((size_t)h * a.max_seq + pos) * 2 * a.hd + a.hd + e;
                    dst[0] = v0;
                    dst[1] = v1;
                }
            }
        }
    }
}

// Repack upstream AoS Q4_0 blocks ([M][nb] x 20 B) into stream tiles.
// interleave_half != 0: destination row 2i takes source row i and 2i+1 takes
// source row interleave_half + i (gate/up pairing).
__global__ void q4_pack_kernel(const uint8_t* __restrict__ src, uint32_t M, uint32_t K,
                               uint32_t R, uint32_t interleave_half, uint8_t* __restrict__ dst) {
    const uint32_t nb = K / 32;
    const uint64_t n = (uint64_t)M * nb;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t drow = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
        uint32_t srow = drow;
        if (interleave_half) srow = (drow & 1) ? interleave_half + drow / 2 : drow / 2;
        const uint32_t* s = reinterpret_cast<const uint32_t*>(src + ((size_t)srow * nb + b) * 20);
        const uint32_t tile = drow / R, r = drow % R;
        uint8_t* tb = dst + (size_t)tile * gemv_tile_bytes(R, K);
        uint4 q = make_uint4(s[0], s[1], s[2], s[3]);
        *reinterpret_cast<uint4*>(tb + ((size_t)r * nb + b) * 16) = q;
        *reinterpret_cast<uint32_t*>(tb + (size_t)R * nb * 16 + ((size_t)r * nb + b) * 4) = s[4];
    }
}

}  // namespace qb200
