// sample.cuh — stochastic token sampling on the device (temperature, top-k,
// top-p), so a generation loop never copies logits to the host.
//
// Restates upstream q_sample_token (src/main.c:852-991) and its helpers:
//   compute_softmax_with_temp (main.c:311-424): logits * (1 / T) on the
//     8-wide vector body, logits / T on the tail, then q_softmax_f32_avx2
//     (softmax.c: the clamped polynomial exp below 8 floor(V/8), expf on the
//     tail, out = e * (1 / sum)); logits that are not 32-byte aligned are
//     divided by T everywhere, as upstream's unaligned temperature loop does
//     (its softmax then still runs on its own aligned arena buffer).  With a
//     NULL context upstream's buffer comes from malloc and its alignment picks
//     between the two softmax forms at random; this follows the arena case,
//     the one upstream's q_generate takes;
//   apply_top_k (main.c:430-519): the k most probable tokens, renormalised by
//     division by their sum (disabled when k == 0 or k >= V);
//   apply_top_p (main.c:608-716): after sorting by probability, the shortest
//     prefix whose running sum reaches p (all tokens when none does),
//     renormalised the same way (disabled unless 0 < p < 1);
//   the xorshift64* draw (main.c:950-973) and the CDF walk over the kept
//     tokens in index order (main.c:720-760), falling back to the last kept
//     token when rounding leaves the draw above the total.
// Upstream leaves the keep-mask unset when neither filter is on; here every
// token is kept then, which is what that code path intends.  Ties: upstream
// selects among equal probabilities by quicksort order (unspecified); here
// the lower index wins.
//
// One CTA of 1024 threads.  Thresholds come from 4-pass radix selection on
// the (non-negative) float bits; the bucket sums top-p needs are added as
// 2^-52 fixed-point integers so every run gives the same bits.
#pragma once

#include "common.cuh"

namespace qb200 {

static constexpr uint32_t SAMPLE_THREADS = 1024;

struct SampleParams {  // device-resident, read by the kernel on every launch
    float temperature;  // < 1e-6: greedy (the kernel leaves the argmax key alone)
    uint32_t top_k;
    float top_p;
    uint32_t scalar_path;  // unaligned logits: divide by T everywhere (upstream's scalar loop)
};

struct SampleArgs {
    const float* logits;             // [V]
    uint32_t V;
    const SampleParams* params;
    unsigned long long* rng;         // xorshift64* state (advanced once per launch)
    float* probs;                    // scratch [V]
    uint8_t* keep;                   // scratch [V]
    unsigned long long* best;        // out: the chosen token in the argmax-key encoding
    uint32_t* token_out;             // optional out: the token
};

__device__ __forceinline__ float block_sum_1024(float v, float* red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    if (warp == 0) {
        t = red[lane];
        t = warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

__device__ __forceinline__ float block_max_1024(float v, float* red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = warp_max(red[lane]);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// Exclusive prefix over the block (thread order) of per-thread values.
template <typename T>
__device__ __forceinline__ T block_excl_scan_1024(T v, T* buf, T& total) {
    const uint32_t tid = threadIdx.x;
    __syncthreads();
    buf[tid] = v;
    __syncthreads();
    for (uint32_t off = 1; off < SAMPLE_THREADS; off <<= 1) {
        T add = tid >= off ? buf[tid - off] : T(0);
        __syncthreads();
        buf[tid] += add;
        __syncthreads();
    }
    total = buf[SAMPLE_THREADS - 1];
    const T incl = buf[tid];
    __syncthreads();
    return incl - v;
}

// k-th largest key (k >= 1) among keys of kept elements: radix selection on
// 32-bit keys, 8 bits per pass.  Returns the key; *n_gt = kept elements with
// a larger key.  Keys of non-negative floats order like the floats.
__device__ inline uint32_t radix_kth_largest(const float* p, const uint8_t* keep, uint32_t V, uint32_t k,
                                             uint32_t* hist, uint32_t* n_gt) {
    const uint32_t tid = threadIdx.x;
    uint32_t prefix = 0, mask = 0, above = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t b = tid; b < 256; b += SAMPLE_THREADS) hist[b] = 0;
        __syncthreads();
        for (uint32_t i = tid; i < V; i += SAMPLE_THREADS) {
            if (keep && !keep[i]) continue;
            const uint32_t key = __float_as_uint(p[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        __shared__ uint32_t s_digit, s_above;
        if (tid == 0) {
            uint32_t acc = above, d = 0;
            for (int b = 255; b >= 0; --b) {
                if (acc + hist[b] >= k) {
                    d = (uint32_t)b;
                    break;
                }
                acc += hist[b];
            }
            s_digit = d;
            s_above = acc;
        }
        __syncthreads();
        prefix |= s_digit << shift;
        mask |= 255u << shift;
        above = s_above;
        __syncthreads();
    }
    *n_gt = above;
    return prefix;
}

__global__ void __launch_bounds__(SAMPLE_THREADS, 1) sample_kernel(const SampleArgs a) {
    __shared__ float red[33];
    __shared__ uint32_t hist[256];
    __shared__ unsigned long long hsum[256];
    __shared__ uint32_t scan_u[SAMPLE_THREADS];
    __shared__ float scan_f[SAMPLE_THREADS];
    pdl_wait();
    const SampleParams prm = *a.params;
    if (!(prm.temperature >= 1e-6f)) return;  // greedy: the head's argmax key stands
    const uint32_t tid = threadIdx.x, V = a.V;
    const uint32_t nv = V / 8 * 8;  // upstream's vector body (multiply by 1/T, poly exp)
    float* p = a.probs;
    // ---- softmax with temperature ----
    const float T = prm.temperature, inv_t = __fdiv_rn(1.0f, T);
    float mx = -INFINITY;
    for (uint32_t i = tid; i < V; i += SAMPLE_THREADS) {
        const float l = a.logits[i];
        const float s = (!prm.scalar_path && i < nv) ? __fmul_rn(l, inv_t) : __fdiv_rn(l, T);
        p[i] = s;
        mx = fmaxf(mx, s);
    }
    mx = block_max_1024(mx, red);
    float sum = 0.0f;
    for (uint32_t i = tid; i < V; i += SAMPLE_THREADS) {
        const float x = __fsub_rn(p[i], mx);
        const float e = i < nv ? exp_poly(x) : expf(x);
        p[i] = e;
        sum += e;
    }
    sum = block_sum_1024(sum, red);
    const float inv = __fdiv_rn(1.0f, sum);
    for (uint32_t i = tid; i < V; i += SAMPLE_THREADS) {
        p[i] = sum > 0.0f ? __fmul_rn(p[i], inv) : __fdiv_rn(1.0f, (float)V);
        a.keep[i] = 1;
    }
    __syncthreads();
    // per-thread contiguous ranges for the order-dependent steps
    const uint32_t chunk = (V + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
    const uint32_t c0 = min(V, tid * chunk), c1 = min(V, c0 + chunk);
    // ---- top-k ----
    if (prm.top_k > 0 && prm.top_k < V) {
        uint32_t n_gt = 0;
        const uint32_t key = radix_kth_largest(p, nullptr, V, prm.top_k, hist, &n_gt);
        const uint32_t m = prm.top_k - n_gt;  // ties at the threshold, lowest index first
        uint32_t eq = 0;
        for (uint32_t i = c0; i < c1; ++i) eq += __float_as_uint(p[i]) == key;
        uint32_t tot;
        uint32_t before = block_excl_scan_1024<uint32_t>(eq, scan_u, tot);
        float s = 0.0f;
        for (uint32_t i = c0; i < c1; ++i) {
            const uint32_t kb = __float_as_uint(p[i]);
            bool k8 = kb > key;
            if (kb == key) k8 = before++ < m;
            a.keep[i] = k8;
            if (k8) s += p[i];
        }
        s = block_sum_1024(s, red);
        for (uint32_t i = c0; i < c1; ++i) p[i] = a.keep[i] && s > 0.0f ? __fdiv_rn(p[i], s) : (s > 0.0f ? 0.0f : p[i]);
        __syncthreads();
    }
    // ---- top-p ----
    if (prm.top_p > 0.0f && prm.top_p < 1.0f) {
        const double fx = 4503599627370496.0;  // 2^52
        const unsigned long long target = (unsigned long long)((double)prm.top_p * fx);
        uint32_t prefix = 0, mask = 0;
        unsigned long long acc = 0;
        bool reached = true;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (uint32_t b = tid; b < 256; b += SAMPLE_THREADS) {
                hist[b] = 0;
                hsum[b] = 0ull;
            }
            __syncthreads();
            for (uint32_t i = tid; i < V; i += SAMPLE_THREADS) {
                const uint32_t kb = __float_as_uint(p[i]);
                if ((kb & mask) == prefix) {
                    const uint32_t b = (kb >> shift) & 255u;
                    atomicAdd(&hist[b], 1u);
                    atomicAdd(&hsum[b], (unsigned long long)((double)p[i] * fx));
                }
            }
            __syncthreads();
            __shared__ uint32_t s_digit, s_reached;
            __shared__ unsigned long long s_acc;
            if (tid == 0) {
                unsigned long long t = acc;
                int d = -1;
                for (int b = 255; b >= 0; --b) {
                    if (hist[b] && t + hsum[b] >= target) {
                        d = b;
                        break;
                    }
                    t += hsum[b];
                }
                s_reached = d >= 0;
                s_digit = d >= 0 ? (uint32_t)d : 0u;
                s_acc = t;
            }
            __syncthreads();
            if (!s_reached) {
                reached = false;
                break;
            }
            prefix |= s_digit << shift;
            mask |= 255u << shift;
            acc = s_acc;
            __syncthreads();
        }
        // keep every token above the threshold value, and of the tokens equal
        // to it the first m (index order) with acc + m * value >= top_p
        const float tv = __uint_as_float(prefix);
        uint32_t m = 0xFFFFFFFFu;
        if (reached && tv > 0.0f) {
            const double need = ((double)target - (double)acc) / fx;
            m = (uint32_t)max(1.0, ceil(need / (double)tv));
        }
        uint32_t eq = 0;
        for (uint32_t i = c0; i < c1; ++i) eq += __float_as_uint(p[i]) == prefix;
        uint32_t tot;
        uint32_t before = block_excl_scan_1024<uint32_t>(eq, scan_u, tot);
        float s = 0.0f;
        for (uint32_t i = c0; i < c1; ++i) {
            bool k8 = true;  // the running sum never reaches p: every token
            if (reached && tv > 0.0f) {
                const uint32_t kb = __float_as_uint(p[i]);
                k8 = kb > prefix;
                if (kb == prefix) k8 = before++ < m;
            }
            a.keep[i] = k8;
            if (k8) s += p[i];
        }
        s = block_sum_1024(s, red);
        for (uint32_t i = c0; i < c1; ++i) p[i] = a.keep[i] && s > 0.0f ? __fdiv_rn(p[i], s) : (s > 0.0f ? 0.0f : p[i]);
        __syncthreads();
    }
    // ---- the draw (upstream xorshift64*, one per call) ----
    __shared__ float s_r;
    if (tid == 0) {
        unsigned long long x = *a.rng;
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        *a.rng = x;
        const uint32_t u = (uint32_t)((x * 0x2545F4914F6CDD1DULL) >> 32);
        s_r = (float)(u >> 8) / 16777216.0f;
    }
    __syncthreads();
    const float r = s_r;
    // ---- CDF walk over the kept tokens in index order ----
    float part = 0.0f;
    for (uint32_t i = c0; i < c1; ++i)
        if (a.keep[i]) part += p[i];
    float total;
    float run = block_excl_scan_1024<float>(part, scan_f, total);
    __shared__ uint32_t s_pick;
    if (tid == 0) s_pick = 0xFFFFFFFFu;
    __syncthreads();
    for (uint32_t i = c0; i < c1; ++i) {
        if (!a.keep[i]) continue;
        run += p[i];
        if (r < run) {
            atomicMin(&s_pick, i);
            break;
        }
    }
    __syncthreads();
    uint32_t last = 0;
    for (uint32_t i = c0; i < c1; ++i)
        if (a.keep[i]) last = max(last, i + 1);
    __shared__ uint32_t s_last;
    if (tid == 0) s_last = 0;
    __syncthreads();
    atomicMax(&s_last, last);
    __syncthreads();
    if (tid == 0) {
        uint32_t tok = s_pick;
        if (tok == 0xFFFFFFFFu) tok = s_last ? s_last - 1 : V - 1;  // rounding left r above the total
        *a.best = (1ull << 32) | (unsigned long long)(0xFFFFFFFFu - tok);
        if (a.token_out) *a.token_out = tok;
    }
}

}  // namespace qb200
