// ops.cuh — standalone device kernels behind the upstream kernel-level entry
// points (q_rmsnorm_f32_avx2, q_rope_f32_avx2, q_silu_f32_avx2,
// q_softmax_f32_avx2, q_add/mul_f32_avx2, q_causal_mask_f32_avx2,
// q_matmul_f32_avx2, q_dequantize_q4_0_block_avx2_public).  The model
// forward does not use these: it runs the same arithmetic fused into the
// GEMV / attention kernels.  They exist so code written against upstream's
// kernel API runs on the device unchanged.
#pragma once

#include "common.cuh"

namespace qb200 {

static constexpr int OPS_THREADS = 256;

// upstream rmsnorm.c:15-92 (one CTA)
__global__ void rmsnorm_kernel(const float* x, const float* w, float* out, uint32_t n, float eps) {
    __shared__ float part[OPS_THREADS / 32];
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += OPS_THREADS) ss = __fmaf_rn(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < OPS_THREADS / 32; ++i) tot += part[i];
    float me = __fadd_rn(__fdiv_rn(tot, (float)n), eps);
    float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
    float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
    float r = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
    for (uint32_t i = threadIdx.x; i < n; i += OPS_THREADS) out[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
}

// upstream rope.c:23-110
__global__ void rope_kernel(const float* x, const float* c, const float* s, float* out, uint32_t n) {
    const uint32_t i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i + 1 >= n) return;
    out[i] = __fsub_rn(__fmul_rn(x[i], c[i]), __fmul_rn(x[i + 1], s[i]));
    out[i + 1] = __fadd_rn(__fmul_rn(x[i + 1], c[i + 1]), __fmul_rn(x[i], s[i + 1]));
}

// upstream silu.c:18-94: polynomial exp on i < 8*floor(n/8) (none when n < 8)
__global__ void silu_kernel(const float* x, float* out, uint32_t n) {
    const uint32_t nv = n < 8 ? 0u : n / 8 * 8;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (i < nv) {
            out[i] = silu_poly(x[i]);
        } else {
            const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x[i])));
            out[i] = __fmul_rn(x[i], sg);
        }
    }
}

// upstream softmax.c:17-132 (one CTA)
__global__ void softmax_kernel(const float* x, float* out, uint32_t n) {
    __shared__ float part[OPS_THREADS / 32];
    __shared__ float bc;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += OPS_THREADS) m = fmaxf(m, x[i]);
    m = warp_max(m);
    if (lane == 0) part[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = -INFINITY;
        for (int i = 0; i < OPS_THREADS / 32; ++i) t = fmaxf(t, part[i]);
        bc = t;
    }
    __syncthreads();
    m = bc;
    const uint32_t nv = n < 8 ? 0u : n / 8 * 8;
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += OPS_THREADS) {
        const float d = __fsub_rn(x[i], m);
        const float e = i < nv ? exp_poly(d) : expf(d);
        out[i] = e;
        s += e;
    }
    s = warp_sum(s);
    __syncthreads();
    if (lane == 0) part[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < OPS_THREADS / 32; ++i) t += part[i];
        bc = t;
    }
    __syncthreads();
    s = bc;
    if (n < 8) {
        for (uint32_t i = threadIdx.x; i < n; i += OPS_THREADS) out[i] = __fdiv_rn(out[i], s);
    } else {
        const float inv = __fdiv_rn(1.0f, s);
        for (uint32_t i = threadIdx.x; i < n; i += OPS_THREADS) out[i] = __fmul_rn(out[i], inv);
    }
}

// op 0: add, 1: mul (upstream add_fp32.c / mul_fp32.c; aliasing allowed)
__global__ void binary_kernel(const float* a, const float* b, float* o, uint32_t n, int op) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        o[i] = op ? __fmul_rn(a[i], b[i]) : __fadd_rn(a[i], b[i]);
}

// upstream causal_mask_fp32.c: scores[i][j] = mask for j > i (row stride ld)
__global__ void causal_mask_kernel(float* s, uint32_t n, size_t ld, float mask) {
    for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < (uint64_t)n * n;
         k += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t i = (uint32_t)(k / n), j = (uint32_t)(k % n);
        if (j > i) s[(size_t)i * ld + j] = mask;
    }
}

// C[M,N] = A[M,K] B[K,N] with arbitrary element strides (small matrices)
__global__ void matmul_f32_kernel(const float* A, size_t sar, size_t sac, const float* B,
                                  size_t sbr, size_t sbc, float* C, size_t scr, uint32_t M,
                                  uint32_t N, uint32_t K) {
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < (uint64_t)M * N;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t i = (uint32_t)(t / N), j = (uint32_t)(t % N);
        float acc = 0.0f;
        for (uint32_t k = 0; k < K; ++k) acc = __fmaf_rn(A[i * sar + k * sac], B[k * sbr + j * sbc], acc);
        C[(size_t)i * scr + j] = acc;
    }
}

// upstream dequantize.c:18-73: w = fma(q, s, -8 s)
__global__ void dequant_block_kernel(const uint8_t* blk, float* out) {
    const uint32_t i = threadIdx.x;
    if (i >= 32) return;
    float s;
    memcpy(&s, blk + 16, 4);
    const uint8_t b = blk[i / 2];
    const float q = (float)((i & 1) ? (b >> 4) : (b & 15));
    out[i] = __fmaf_rn(q, s, __fmul_rn(-8.0f, s));
}

}  // namespace qb200
