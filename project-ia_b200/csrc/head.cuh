// head.cuh — final RMSNorm + FP32 LM head + greedy argmax, and the
// per-step bookkeeping kernel (sm_100a).
//
// Replaces upstream model.c:1799-1844 (rmsnorm of the last row, then
// q_matmul_f32_avx2 against the transposed FP32 output view) and the greedy
// branch of q_sample_token (src/main.c:870-881: the first index of the
// maximum).  The head streams W_out [V][D] fp32 (2.1 GB at the 8B shape)
// through a shared-memory ring by bulk copies, x normalised once per CTA
// into shared memory, packed FFMA2 accumulation, and folds the argmax into a 64-bit
// atomicMax over (order-preserving float bits, ~index) so ties resolve to
// the lowest index exactly like upstream's strict '>' scan.
#pragma once

#include "common.cuh"
#include "gemv_q4.cuh"

namespace qb200 {

static constexpr int HEAD_CWARPS = 8;                            // consumer warps
static constexpr int HEAD_THREADS = HEAD_CWARPS * 32 + 32;         // + producer warp
static constexpr uint32_t HEAD_STAGE_BYTES = 64 * 1024;            // one ring slot
static constexpr uint32_t HEAD_MAX_SLOTS = 3;
static constexpr uint32_t HEAD_MAX_PARTS = 8;                      // warps sharing one row
static constexpr uint32_t HEAD_MAX_ROWS_PER_STAGE = 32;

struct HeadArgs {
    const float* w;            // [rows][K] fp32
    const float* x;            // residual stream [K]
    const float* norm_w;       // final norm gains (null: no norm)
    float eps;
    uint32_t rows, K;
    uint32_t row_base;         // global index of row 0 (vocab split)
    uint32_t slots;            // ring depth (2..HEAD_MAX_SLOTS)
    float* logits;             // [rows]
    unsigned long long* best;  // argmax key (null: none)
    unsigned long long* trace; // step-trace slot (null: off)
    // Tensor-parallel exchange (peer memory; see GemvTp):
    //   tp.tp_recv: x is not read; the input is the rank-order sum of the W
    //   slots of parity tp.tp_par that the last layer's down projection sent,
    //   and CTA 0 stores that sum (the residual stream) to x_copy;
    //   tp_key: once every CTA has folded its rows into *best (local ticket),
    //   the last CTA stores the key as key word[rank][0..1] of every rank (low
    //   and high halves, each tagged with the key exchange's sequence number);
    //   advance_kernel takes the maximum of the W keys.
    GemvTp tp;
    float* x_copy;
    uint32_t tp_key;
};

// Shared memory: ring[slots][HEAD_STAGE_BYTES] | x[K] fp32.
__host__ __device__ inline size_t head_smem_bytes(uint32_t K, uint32_t slots) {
    return (size_t)slots * HEAD_STAGE_BYTES + (size_t)K * 4;
}

// Ring depth for K: as many 64 KB slots (2..3) as fit beside x in the
// 220 KB budget; 0 when K is out of range (K % 4, K * 4 > one slot).
inline uint32_t head_slots(uint32_t K) {
    if (K == 0 || K % 4 || (size_t)K * 4 > HEAD_STAGE_BYTES) return 0;
    for (uint32_t sl = HEAD_MAX_SLOTS; sl >= 2; --sl)
        if (head_smem_bytes(K, sl) <= 220 * 1024) return sl;
    return 0;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - idx);
}

// One CTA per SM over a contiguous range of rows.  The producer warp
// streams the range through the ring in stages of whole rows (one 1-D bulk
// copy per stage, this GPU's own memory, no multicast), starting before the
// programmatic-dependency wait since the weights do not depend on the
// previous kernel.  The consumer warps split each stage into (row, part)
// items — a row in P = 8 / rows-per-stage parts — take items round-robin,
// and leave one partial per item in shared memory; the row's logit is the
// sum of its P partials in part order.  Requires K * 4 <= HEAD_STAGE_BYTES
// and K % 4 == 0 (host-checked).
__global__ void __launch_bounds__(HEAD_THREADS, 1) lm_head_kernel(const HeadArgs a) {
    extern __shared__ __align__(128) uint8_t hsm[];
    constexpr uint32_t T = HEAD_CWARPS * 32;
    __shared__ __align__(8) uint64_t full[HEAD_MAX_SLOTS], empty[HEAD_MAX_SLOTS];
    __shared__ float part[HEAD_CWARPS];
    __shared__ float red[HEAD_MAX_ROWS_PER_STAGE > HEAD_MAX_PARTS ? HEAD_MAX_ROWS_PER_STAGE : HEAD_MAX_PARTS];  // [row in stage][part]
    __shared__ unsigned long long wbest[HEAD_CWARPS];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = a.K, rb = K * 4, SR = min(HEAD_MAX_ROWS_PER_STAGE, HEAD_STAGE_BYTES / rb);  // rows per stage
    const uint32_t P = SR >= HEAD_CWARPS ? 1u : HEAD_CWARPS / SR;      // parts per row
    const uint32_t r0 = (uint32_t)((uint64_t)a.rows * blockIdx.x / gridDim.x);
    const uint32_t r1 = (uint32_t)((uint64_t)a.rows * (blockIdx.x + 1) / gridDim.x);
    float* xs = reinterpret_cast<float*>(hsm + (size_t)a.slots * HEAD_STAGE_BYTES);
    if (tid == 0) {
        trace_mark(a.trace, 0);
        for (uint32_t s = 0; s < a.slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], HEAD_CWARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == HEAD_CWARPS) {
        // ---- producer ---------------------------------------------------------------
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t s = 0, ph = 0, k = 0;
            for (uint32_t row = r0; row < r1; row += SR, ++k) {
                if (k >= a.slots && !mbar_wait(&empty[s], ph ^ 1, QDEV_WAIT_EMPTY_TIMEOUT)) break;
                const uint32_t bytes = min(SR, r1 - row) * rb;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(hsm + (size_t)s * HEAD_STAGE_BYTES, a.w + (size_t)row * K, bytes, &full[s], pol);
                if (++s == a.slots) {
                    s = 0;
                    ph ^= 1;
                }
            }
        }
        pdl_wait();  // every thread waits: the grid ends after its predecessor
        return;
    }

    // ---- consumers: normalised x into shared memory ------------------------------------
    pdl_wait();
    if (tid == 0) trace_mark(a.trace, 1);
    if (a.tp.tp_recv) {
        // the W slots in rank order, as the one-shot all-reduce adds them
        const uint32_t want = __ldcg(tp_ctl(a.tp, a.tp.tp_rank) + 2 + a.tp.tp_par) + 1u;
        const unsigned long long t0 = gtimer();
        bool late = false;
        constexpr int NR = 4;
        const uint32_t n4 = K / 4;
        for (uint32_t base = 0; base < n4; base += T * NR) {
            float4 xv[NR];
            tp_take_all<NR>(a.tp, base, tid, T, n4, want, xv, t0, late);
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint32_t i = base + tid + T * r;
                if (i < n4) {
                    reinterpret_cast<float4*>(xs)[i] = xv[r];
                    if (a.x_copy && blockIdx.x == 0) reinterpret_cast<float4*>(a.x_copy)[i] = xv[r];
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        if (tid == 0) tp_recv_done(a.tp, want);
    } else {
        for (uint32_t i = tid; i < K; i += T) xs[i] = a.x[i];
    }
    // (without a receive each thread normalises the elements it stored, so
    // no barrier is needed yet)
    float r = 1.0f;
    if (a.norm_w) {
        float ss = 0.0f;
        for (uint32_t i = tid; i < K; i += T) ss = __fmaf_rn(xs[i], xs[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) part[warp] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        float tot = 0.0f;
        for (int i = 0; i < HEAD_CWARPS; ++i) tot += part[i];
        float me = __fadd_rn(__fdiv_rn(tot, (float)K), a.eps);
        float r0f = __fdiv_rn(1.0f, __fsqrt_rn(me));
        float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0f, r0f)));
        r = __fmul_rn(__fmul_rn(r0f, tm), 0.5f);
    }
    if (a.norm_w)
        for (uint32_t i = tid; i < K; i += T) xs[i] = __fmul_rn(__fmul_rn(xs[i], r), a.norm_w[i]);
    asm volatile("bar.sync 1, %0;" ::"r"(T));

    // ---- consumers: stages ----------------------------------------------------------
    const uint32_t n4 = K / 4, pl4 = (n4 + P - 1) / P;  // float4s per part
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    unsigned long long best = 0ull;
    uint32_t s = 0, ph = 0;
    for (uint32_t row = r0; row < r1; row += SR) {
        const uint32_t nr = min(SR, r1 - row);
        mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
        const float4* st4 = reinterpret_cast<const float4*>(hsm + (size_t)s * HEAD_STAGE_BYTES);
        for (uint32_t it = warp; it < nr * P; it += HEAD_CWARPS) {
            const uint32_t rr = it / P, p = it % P;
            const uint32_t b = p * pl4, e = min(n4, b + pl4);
            const float4* wr = st4 + (size_t)rr * n4;
            float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
            uint32_t i = b + lane;
            for (; i + 32 < e; i += 64) {
                const float4 w0 = wr[i], w1 = wr[i + 32], xa = x4[i], xb = x4[i + 32];
                acc0 = __ffma2_rn(make_float2(w0.x, w0.y), make_float2(xa.x, xa.y), acc0);
                acc0 = __ffma2_rn(make_float2(w0.z, w0.w), make_float2(xa.z, xa.w), acc0);
                acc1 = __ffma2_rn(make_float2(w1.x, w1.y), make_float2(xb.x, xb.y), acc1);
                acc1 = __ffma2_rn(make_float2(w1.z, w1.w), make_float2(xb.z, xb.w), acc1);
            }
            if (i < e) {
                const float4 w0 = wr[i], xa = x4[i];
                acc0 = __ffma2_rn(make_float2(w0.x, w0.y), make_float2(xa.x, xa.y), acc0);
                acc0 = __ffma2_rn(make_float2(w0.z, w0.w), make_float2(xa.z, xa.w), acc0);
            }
            const float d = warp_sum((acc0.x + acc0.y) + (acc1.x + acc1.y));
            if (lane == 0) red[rr * P + p] = d;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == a.slots) {
            s = 0;
            ph ^= 1;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        if (tid < nr) {
            float d = 0.0f;
            for (uint32_t p = 0; p < P; ++p) d += red[tid * P + p];
            a.logits[row + tid] = d;
            const unsigned long long kk = argmax_key(d, a.row_base + row + tid);
            best = kk > best ? kk : best;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(T));  // red[] free again
    }
    if (!a.best) {
        if (tid == 0) trace_mark(a.trace, 2);
        return;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    if (lane == 0) wbest[warp] = best;
    asm volatile("bar.sync 1, %0;" ::"r"(T));
    if (tid == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < HEAD_CWARPS; ++i) b = wbest[i] > b ? wbest[i] : b;
        if (b) atomicMax(a.best, b);
        if (a.tp_key) {
            uint32_t* ctl = tp_ctl(a.tp, a.tp.tp_rank);
            uint32_t old;
            __threadfence();
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                         : "=r"(old)
                         : "l"(ctl + TP_CTL_HEAD_TICKET)
                         : "memory");
            if (old == gridDim.x - 1) {  // every CTA's key is folded in
                ctl[TP_CTL_HEAD_TICKET] = 0u;
                const unsigned long long k = atomicAdd(a.best, 0ull);
                const uint32_t seq = __ldcg(ctl + TP_CTL_KEY_SEQ) + 1u;
                for (uint32_t q = 0; q < a.tp.tp_world; ++q) {
                    uint64_t* kw = reinterpret_cast<uint64_t*>(tp_ctl(a.tp, q) + TP_CTL_KEY) + 2 * a.tp.tp_rank;
                    st_relaxed_sys_u64(kw, ((uint64_t)seq << 32) | (uint32_t)k);
                    st_relaxed_sys_u64(kw + 1, ((uint64_t)seq << 32) | (uint32_t)(k >> 32));
                }
            }
        }
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
    uint32_t* key_ctl;         // tensor parallel: this rank's exchange control words (null: *best alone)
    uint32_t key_world;
};

__global__ void advance_kernel(const AdvanceArgs a) {
    if (threadIdx.x == 0) trace_mark(a.trace, 0);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    trace_mark(a.trace, 1);
    unsigned long long k = *a.best;
    if (a.key_ctl) {  // the maximum of every rank's key (the LM head's tp_key exchange)
        const uint32_t want = __ldcg(a.key_ctl + TP_CTL_KEY_SEQ) + 1u;
        const unsigned long long t0 = gtimer(), lim = qdev_wait_ns();
        k = 0ull;
        const uint64_t* kw = reinterpret_cast<const uint64_t*>(a.key_ctl + TP_CTL_KEY);
        for (uint32_t q = 0; q < a.key_world; ++q) {
            ulonglong2 w = ld_relaxed_sys_u64x2(kw + 2 * q);
            while ((uint32_t)(w.x >> 32) != want || (uint32_t)(w.y >> 32) != want) {
                if (gtimer() - t0 > lim) {
                    qdev_fail(QDEV_PEER_TIMEOUT);
                    break;
                }
                w = ld_relaxed_sys_u64x2(kw + 2 * q);
            }
            const unsigned long long v = ((unsigned long long)(uint32_t)w.y << 32) | (uint32_t)w.x;
            k = v > k ? v : k;
        }
        __stcg(a.key_ctl + TP_CTL_KEY_SEQ, want);
    }
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
