// head.cuh — final RMSNorm + FP32 LM head + greedy argmax, and the
// per-step bookkeeping kernel (sm_100a).
//
// Replaces upstream model.c:1799-1844 (rmsnorm of the last row, then
// q_matmul_f32_avx2 against the transposed FP32 output view) and the greedy
// branch of q_sample_token (src/main.c:870-881: the first index of the
// maximum).  The head streams W_out [V][D] fp32 (2.1 GB at the 8B shape)
// with 16-byte non-allocating loads, x normalised once per CTA into shared
// memory, packed FFMA2 accumulation, and folds the argmax into a 64-bit
// atomicMax over (order-preserving float bits, ~index) so ties resolve to
// the lowest index exactly like upstream's strict '>' scan.
#pragma once

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

static constexpr int HEAD_THREADS = 256;

struct HeadArgs {
    const float* w;            // [rows][K] fp32
    const float* x;            // residual stream [K]
    const float* norm_w;       // final norm gains (null: no norm)
    float eps;
    uint32_t rows, K;
    uint32_t row_base;         // global index of row 0 (vocab split)
    float* logits;             // [rows]
    unsigned long long* best;  // argmax key (null: none)
    unsigned long long* trace; // step-trace slot (null: off)
};

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - idx);
}

__global__ void __launch_bounds__(HEAD_THREADS) lm_head_kernel(const HeadArgs a) {
    extern __shared__ __align__(16) float xs[];  // [K]
    __shared__ float part[HEAD_THREADS / 32];
    __shared__ unsigned long long wbest[HEAD_THREADS / 32];
    if (threadIdx.x == 0) trace_mark(a.trace, 0);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(a.trace, 1);
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float r = 1.0f;
    if (a.norm_w) {
        float ss = 0.0f;
        for (uint32_t i = tid; i < a.K; i += HEAD_THREADS) ss = __fmaf_rn(a.x[i], a.x[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) part[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int i = 0; i < HEAD_THREADS / 32; ++i) tot += part[i];
        float me = __fadd_rn(__fdiv_rn(tot, (float)a.K), a.eps);
        float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
        float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
        r = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
    }
    for (uint32_t i = tid; i < a.K; i += HEAD_THREADS)
        xs[i] = a.norm_w ? __fmul_rn(__fmul_rn(a.x[i], r), a.norm_w[i]) : a.x[i];
    __syncthreads();

    const uint32_t nw = gridDim.x * (HEAD_THREADS / 32);
    const uint32_t gw = blockIdx.x * (HEAD_THREADS / 32) + warp;
    const uint32_t n4 = a.K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    unsigned long long best = 0ull;
    for (uint32_t row = gw * 2; row < a.rows; row += nw * 2) {
        const bool two = row + 1 < a.rows;
        const float4* w0 = reinterpret_cast<const float4*>(a.w + (size_t)row * a.K);
        const float4* w1 = reinterpret_cast<const float4*>(a.w + (size_t)(two ? row + 1 : row) * a.K);
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
        float2 acc2 = make_float2(0.f, 0.f), acc3 = make_float2(0.f, 0.f);
        uint32_t i = lane;
        for (; i + 32 < n4; i += 64) {
            const float4 a0 = ldg_stream_f4(w0 + i), a1 = ldg_stream_f4(w0 + i + 32);
            const float4 b0 = ldg_stream_f4(w1 + i), b1 = ldg_stream_f4(w1 + i + 32);
            const float4 xa = x4[i], xb = x4[i + 32];
            acc0 = __ffma2_rn(make_float2(a0.x, a0.y), make_float2(xa.x, xa.y), acc0);
            acc0 = __ffma2_rn(make_float2(a0.z, a0.w), make_float2(xa.z, xa.w), acc0);
            acc1 = __ffma2_rn(make_float2(a1.x, a1.y), make_float2(xb.x, xb.y), acc1);
            acc1 = __ffma2_rn(make_float2(a1.z, a1.w), make_float2(xb.z, xb.w), acc1);
            acc2 = __ffma2_rn(make_float2(b0.x, b0.y), make_float2(xa.x, xa.y), acc2);
            acc2 = __ffma2_rn(make_float2(b0.z, b0.w), make_float2(xa.z, xa.w), acc2);
            acc3 = __ffma2_rn(make_float2(b1.x, b1.y), make_float2(xb.x, xb.y), acc3);
            acc3 = __ffma2_rn(make_float2(b1.z, b1.w), make_float2(xb.z, xb.w), acc3);
        }
        for (; i < n4; i += 32) {
            const float4 a0 = ldg_stream_f4(w0 + i), b0 = ldg_stream_f4(w1 + i);
            const float4 xa = x4[i];
            acc0 = __ffma2_rn(make_float2(a0.x, a0.y), make_float2(xa.x, xa.y), acc0);
            acc0 = __ffma2_rn(make_float2(a0.z, a0.w), make_float2(xa.z, xa.w), acc0);
            acc2 = __ffma2_rn(make_float2(b0.x, b0.y), make_float2(xa.x, xa.y), acc2);
            acc2 = __ffma2_rn(make_float2(b0.z, b0.w), make_float2(xa.z, xa.w), acc2);
        }
        float d0 = (acc0.x + acc0.y) + (acc1.x + acc1.y);
        float d1 = (acc2.x + acc2.y) + (acc3.x + acc3.y);
        d0 = warp_sum(d0);
        d1 = warp_sum(d1);
        if (lane == 0) {
            a.logits[row] = d0;
            unsigned long long k0 = argmax_key(d0, a.row_base + row);
            best = k0 > best ? k0 : best;
            if (two) {
                a.logits[row + 1] = d1;
                unsigned long long k1 = argmax_key(d1, a.row_base + row + 1);
                best = k1 > best ? k1 : best;
            }
        }
    }
    if (!a.best) {
        if (tid == 0) trace_mark(a.trace, 2);
        return;
    }
    if (lane == 0) wbest[warp] = best;
    __syncthreads();
    if (tid == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < HEAD_THREADS / 32; ++i) b = wbest[i] > b ? wbest[i] : b;
        if (b) atomicMax(a.best, b);
        trace_mark(a.trace, 2);
    }
}

// End of a greedy decode step: publish the argmax as the next token, advance
// the position, clear the argmax key for the next step.
struct AdvanceArgs {
    StepParams* step;
    unsigned long long* best;
    uint32_t* token_out;       // device ring of produced tokens
    uint32_t* token_count;     // index into token_out
    uint32_t token_cap;
    uint32_t* last_token;      // most recent argmax
    unsigned long long* trace; // step-trace slot (null: off)
};

__global__ void advance_kernel(const AdvanceArgs a) {
    if (threadIdx.x == 0) trace_mark(a.trace, 0);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    trace_mark(a.trace, 1);
    const unsigned long long k = *a.best;
    const uint32_t tok = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
    *a.last_token = tok;
    const uint32_t n = *a.token_count;
    if (n < a.token_cap) a.token_out[n] = tok;
    *a.token_count = n + 1;
    StepParams s = *a.step;
    s.token = tok;
    s.pos = s.pos + 1;
    s.n_row = s.pos + 1;
    s.valid = s.pos + 1;
    *a.step = s;
    *a.best = 0ull;
    trace_mark(a.trace, 2);
}

}  // namespace qb200
