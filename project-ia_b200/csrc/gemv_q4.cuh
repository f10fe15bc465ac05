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
// int8 limbs (X = a*65536 + b*256 + c); mma.sync m16n8k32 u8 x s8 -> s32
// multiplies 16 weight rows (q as u8, no float conversion at all) by the
// three limb columns with exact int32 sums, two per 32-row slab sharing the
// limb fragment.  The limbs are recombined and
// the -8*sum(X) term added in fp32, then scaled by s * 2^-(22-e).  The only
// approximations are the 2^-23 (relative to the block max) input grid and
// fp32 accumulation across blocks — the error of an fp32 dot product.
// Versus dequantising to fp32 this needs ~1.4 instead of ~4 instructions
// per weight, so the kernel is HBM-bound rather than issue-bound.
//
// Device weight layout ("slab tiles"): rows in slabs of 32; for each
// (slab, block) 640 bytes: 512 bytes of mma A fragments (lane-major, 16 bytes
// per lane: one word per row g, g+8, g+16, g+24 with g = lane/4, t = lane%4,
// low nibbles = k 4t..4t+3, high nibbles = k 16+4t..16+4t+3) then 32 fp32
// scales laid out [g][rows g, g+8, g+16, g+24].  Blocks of a slab are
// contiguous, slabs follow each other, so any range of blocks is one 1-D
// bulk copy.
//
// Work split.  The grid's CTAs take equal contiguous ranges of the block
// sequence (slab-major), so every CTA streams the same bytes; the host
// prefers a grid that divides the slab count (whole slabs per CTA).  A slab
// cut by a range boundary is finished by the last of its CTAs to arrive
// (per-slab ticket in global scratch), which adds the parts in CTA order.
// Input prologue: coalesced loads staged in shared memory, then one thread
// per 32-value block builds its limb fragment (rows padded to 144 bytes).
// q4_slab_kernel<true> adds the tensor-parallel exchange (GemvTp).
// Inside a CTA a producer warp streams stages through a shared-memory ring
// with cp.async.bulk + mbarrier; weight loads start before the programmatic
// dependent launch wait.  Consumer warp w handles the blocks of a slab with
// index = w (mod warps), so all sums run in a fixed order (deterministic).
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

static constexpr int GEMV_CONSUMER_WARPS = 15;
static constexpr int GEMV_THREADS = GEMV_CONSUMER_WARPS * 32 + 32;
static constexpr uint32_t GEMV_SLAB_ROWS = 32;     // rows per slab (two mma row groups)
static constexpr uint32_t GEMV_BLOCK_BYTES = 640;  // one (slab, block) unit
// x limb fragments of a block: 128 bytes (lanes 0..15; 12..15 zero) in a
// 144-byte row, so that 32 threads writing or reading the same 16-byte
// column of 32 consecutive rows touch every bank (a 128-byte stride would
// put them all on the same four banks).
static constexpr uint32_t GEMV_BFRAG_BYTES = 144;
static constexpr uint32_t GEMV_FSC_BYTES = 32;     // per block: (weight, correction) for t = 0..3
// An RMSNorm prologue needs the whole input in one pass: one 32-value block
// per consumer thread.
static constexpr uint32_t GEMV_MAX_NORM_K = GEMV_CONSUMER_WARPS * 32 * 32;

struct GemvArgs {
    const uint8_t* w;          // packed slab tiles
    uint32_t M, K;             // rows, cols
    uint32_t n_slabs, nb;      // slabs of 32 rows, blocks per row
    uint32_t max_parts;        // CTAs that can share one slab
    const float* x;            // input vector, or the embedding table if gather
    const StepParams* step;    // per-step scalars (token, pos)
    uint32_t gather;           // non-zero: x row = x + step->token * K (embedding)
    const float* norm_w;       // non-null: RMSNorm prologue with these gains
    float eps;
    float* x_copy;             // non-null: CTA 0 stores the raw input here
    float* y;
    const float* resid;
    int epi;
    float* part;               // scratch [n_slabs][max_parts][32]
    uint32_t* ticket;          // scratch [n_slabs], zero between launches
    // EPI_QKV
    const float* rope_cos;     // [max_seq][hd] duplicated-pair tables
    const float* rope_sin;
    float* kv_layer;           // [n_kv][max_seq][2*hd] of this layer
    uint32_t hd, q_rows, kv_rows, max_seq;
};

// Tensor-parallel exchange fused into the GEMVs (peer memory).  Each
// rank's exchange area (at byte tp_off of every rank's buffer) holds
// word[2][W][tp_slice] u64 | control words (256 bytes).  A word is
// (sequence << 32) | fp32 bits, written with one 8-byte store (single-copy
// atomic), so a value and its readiness travel together: the sender needs
// no fence and no flag, the receiver polls the words themselves (the
// low-latency protocol of NCCL's LL transport).  seq[p] in the control
// words is this rank's count of completed receives of parity p; every rank
// runs the same exchanges, so the counts agree.
//   tp_send: the epilogue stores each finished row (plus the residual on the
//   rank whose epilogue adds it) as word[tp_par][rank][row] of every rank,
//   tagged seq[tp_par] + 1, instead of y;
//   tp_recv: every CTA reads the W slots of parity tp_par, waiting (bounded)
//   until each word carries seq[tp_par] + 1, and takes the input as their sum
//   in rank order (the bits a one-shot all-reduce gives); the last CTA done
//   reading (local ticket) advances seq[tp_par].  A slot is written again
//   only by the next exchange of the same parity, whose send follows (in
//   every rank's stream order) the receive of the exchange in between.
struct GemvTp {
    uint8_t* tp_base[8];       // every rank's exchange buffer, mapped here
    uint32_t tp_off, tp_slice, tp_world, tp_rank;
    uint32_t tp_send, tp_recv, tp_par;
};

// Control words (u32 index from the control base): ticket[2] | seq[2] |
// head ticket | key seq | 10 spare | key word[8][2] (u64 at u32 index 16:
// the LM head's argmax key of each rank as two tagged halves).
static constexpr uint32_t TP_CTL_HEAD_TICKET = 4, TP_CTL_KEY_SEQ = 5, TP_CTL_KEY = 16;

__device__ __forceinline__ uint64_t* tp_words(const GemvTp& t, uint32_t rank) {
    return reinterpret_cast<uint64_t*>(t.tp_base[rank] + t.tp_off);
}
__device__ __forceinline__ uint32_t* tp_ctl(const GemvTp& t, uint32_t rank) {
    return reinterpret_cast<uint32_t*>(tp_words(t, rank) + (size_t)2 * t.tp_world * t.tp_slice);
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_relaxed_sys_u64x2(const uint64_t* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t tp_word(uint32_t seq, float v) {
    return ((uint64_t)seq << 32) | __float_as_uint(v);
}

// The input float4s i = base + tid + T r (r < NR, i < n4; zero past n4),
// each the sum over the W received slots in rank order.  For one float4
// the loads of up to 4 slots are issued before any is checked, so a receive
// costs one round trip per float4 a thread takes (two at W = 8), not one
// per rank; a word that is not there yet is polled again until it carries
// `want` or the wait (from t0) runs out — once it has, no later word waits
// (late).
template <int NR>
__device__ __forceinline__ void tp_take_all(const GemvTp& t, uint32_t base, uint32_t tid, uint32_t T, uint32_t n4,
                                            uint32_t want, float4 (&xv)[NR], unsigned long long t0, bool& late) {
    const uint64_t* mine = tp_words(t, t.tp_rank) + (size_t)t.tp_par * t.tp_world * t.tp_slice;
    const uint32_t W = t.tp_world;
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const uint32_t i = base + tid + T * r;
        xv[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i >= n4) continue;
        for (uint32_t q0 = 0; q0 < W; q0 += 4) {  // 4 ranks' loads in flight (registers)
            ulonglong2 w[4][2];
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) {
                if (q0 + k < W) {
                    const uint64_t* p = mine + (size_t)(q0 + k) * t.tp_slice + 4 * (size_t)i;
                    w[k][0] = ld_relaxed_sys_u64x2(p);
                    w[k][1] = ld_relaxed_sys_u64x2(p + 2);
                }
            }
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) {
                const uint32_t q = q0 + k;
                if (q >= W) continue;
                const uint64_t* p = mine + (size_t)q * t.tp_slice + 4 * (size_t)i;
                while (!late && ((uint32_t)(w[k][0].x >> 32) != want || (uint32_t)(w[k][0].y >> 32) != want ||
                                 (uint32_t)(w[k][1].x >> 32) != want || (uint32_t)(w[k][1].y >> 32) != want)) {
                    if (gtimer() - t0 > qdev_wait_ns()) {
                        qdev_fail(QDEV_PEER_TIMEOUT);
                        late = true;
                    } else {
                        w[k][0] = ld_relaxed_sys_u64x2(p);
                        w[k][1] = ld_relaxed_sys_u64x2(p + 2);
                    }
                }
                const float4 v = make_float4(__uint_as_float((uint32_t)w[k][0].x), __uint_as_float((uint32_t)w[k][0].y),
                                             __uint_as_float((uint32_t)w[k][1].x), __uint_as_float((uint32_t)w[k][1].y));
                if (q == 0) {
                    xv[r] = v;
                } else {
                    xv[r].x += v.x;
                    xv[r].y += v.y;
                    xv[r].z += v.z;
                    xv[r].w += v.w;
                }
            }
        }
    }
}

// After every thread of this CTA has read the exchange (call after a CTA
// barrier, one thread): the last CTA of the grid advances the count.
__device__ __forceinline__ void tp_recv_done(const GemvTp& t, uint32_t want) {
    uint32_t* ctl = tp_ctl(t, t.tp_rank);
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctl + t.tp_par) : "memory");
    if (old == gridDim.x - 1) {  // every CTA has read `want` and its words
        ctl[t.tp_par] = 0u;
        __stcg(ctl + 2 + t.tp_par, want);
    }
}

// A chain of up to GEMV_MAX_PHASES GEMVs run by one persistent grid: phase
// p + 1 reads what phase p wrote, so consumers pass a grid barrier between
// phases, while the producer warps stream the next matrices' weights
// straight through it (weights never depend on activations).
static constexpr int GEMV_MAX_PHASES = 4;
struct GemvChain {
    GemvArgs ph[GEMV_MAX_PHASES];
    uint32_t n_phases;
    uint32_t stage_blocks;      // blocks per ring stage
    uint32_t n_stage;           // ring depth
    uint32_t red_slabs;         // slab sums a CTA holds in shared memory between reductions
    uint32_t max_nb;            // largest nb of the phases (input-fragment table size)
    uint32_t* bar;              // n_phases counters, zero between launches (n_phases > 1)
    unsigned long long* trace;  // step-trace slot (null: off)
    GemvTp tp;                  // single-phase launches of q4_slab_kernel<true> only
};

// Shared memory: ring | bfrag[max_nb][144] | fsc[max_nb][4] float2 | red[red_slabs][NW][32] | bars | misc
__host__ __device__ inline size_t gemv_smem_bytes(uint32_t nb, uint32_t stage_blocks,
                                                  uint32_t n_stage, uint32_t red_slabs) {
    return (size_t)n_stage * stage_blocks * GEMV_BLOCK_BYTES + (size_t)nb * GEMV_BFRAG_BYTES +
           (size_t)nb * GEMV_FSC_BYTES + (size_t)red_slabs * GEMV_CONSUMER_WARPS * GEMV_SLAB_ROWS * 4 + 2 * 8 * 8 +
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
template <bool TP>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, const GemvTp& tpa, uint32_t tp_seq, uint32_t j,
                                              uint32_t lane, float v) {
    const float vn = __shfl_down_sync(0xffffffffu, v, 1);
    const uint32_t row = j * GEMV_SLAB_ROWS + lane;
    if (row >= a.M) return;
    if constexpr (TP) {
        if (tpa.tp_send) {  // EPI_STORE / EPI_RESID rows, tagged, to every rank's receive slot
            const float o = a.epi == EPI_RESID ? __fadd_rn(__ldcg(&a.resid[row]), v) : v;
            const size_t at = ((size_t)tpa.tp_par * tpa.tp_world + tpa.tp_rank) * tpa.tp_slice + row;
            const uint64_t w = tp_word(tp_seq, o);
            for (uint32_t r = 0; r < tpa.tp_world; ++r) st_relaxed_sys_u64(tp_words(tpa, r) + at, w);
            return;
        }
    }
    if (a.epi == EPI_STORE) {
        a.y[row] = v;
    } else if (a.epi == EPI_RESID) {
        a.y[row] = __fadd_rn(__ldcg(&a.resid[row]), v);
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

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// This CTA's share of one phase: blocks [x0, x1) of the slab-major
// sequence, its first and last slab, and for those two slabs the lowest and
// highest CTA that holds part of them (equal to this CTA when unshared).
// Computed before the dependency wait: the divisions by the grid size form
// a dependent chain of a few thousand cycles.
struct PhaseRange {
    uint32_t x0, x1, j_first, j_last;
    uint32_t own_lo[2], own_hi[2];  // [first slab, last slab]
};

__device__ inline PhaseRange phase_range(uint32_t n_slabs, uint32_t nb, uint32_t cta, uint32_t G) {
    PhaseRange r;
    const uint32_t NB = n_slabs * nb;
    r.x0 = range_begin(NB, cta, G);
    r.x1 = range_begin(NB, cta + 1, G);
    r.j_first = r.x0 / nb;
    r.j_last = r.x1 > r.x0 ? (r.x1 - 1) / nb : r.j_first;
    r.own_lo[0] = r.own_lo[1] = r.own_hi[0] = r.own_hi[1] = cta;
    if (r.x1 > r.x0) {
        if (r.j_first * nb < r.x0 || (r.j_first + 1) * nb > r.x1) {
            r.own_lo[0] = cta_of(NB, G, r.j_first * nb);
            r.own_hi[0] = cta_of(NB, G, r.j_first * nb + nb - 1);
        }
        if (r.j_last != r.j_first && (r.j_last + 1) * nb > r.x1) r.own_hi[1] = cta_of(NB, G, r.j_last * nb + nb - 1);
    }
    return r;
}

// One GEMV (chain phase) for this CTA's range: input prologue, main loop over
// the ring (slot s / parity ph carried across phases), slab reductions,
// split-slab finish and epilogue.  Consumer threads only (T of them).
template <uint32_t NW, bool TP>
__device__ __forceinline__ void gemv_phase(const GemvArgs& a, const GemvChain& c, uint8_t* smem,
                                           uint8_t* bfrag, float2* fsc, float* red, uint64_t* full,
                                           uint64_t* empty, float* rms_part, uint32_t& s,
                                           uint32_t& ph, uint32_t pidx, bool dry,
                                           const PhaseRange& r) {
    constexpr uint32_t T = NW * 32;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t cta = blockIdx.x;
    const uint32_t nb = a.nb;
    const uint32_t stage_bytes = c.stage_blocks * GEMV_BLOCK_BYTES;
    const uint32_t x0 = r.x0, x1 = r.x1;
    if (x0 >= x1) return;  // (host keeps G <= NB, so never taken)
    const uint32_t j_first = r.j_first, j_last = r.j_last;
    const uint32_t own_lo[2] = {r.own_lo[0], r.own_lo[1]}, own_hi[2] = {r.own_hi[0], r.own_hi[1]};

    // ---- input prologue ------------------------------------------------------------
    const float* xs = a.x;
    if (a.gather) xs = a.x + (size_t)(dry ? 0u : a.step->token) * a.K;
    // Two steps.  (1) Coalesced: thread tid loads float4 number tid + T*r
    // (all loads issued together), applies the RMSNorm, and parks the
    // values in the limb-table area, block b's 128 bytes at the start of
    // its row.  (2) Thread tid converts blocks tid, tid + T, ...: the
    // 32 values of a block in its registers, so the block maximum, the limb
    // bytes and the integer sum need no cross-lane steps; it overwrites the
    // block's own row with the limb fragment.
    const uint32_t nbk = a.K / 32, n4 = a.K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    const float4* g4 = reinterpret_cast<const float4*>(a.norm_w);
    constexpr int NR = 8;
    float r_norm = 1.0f;
    const GemvTp& tpa = c.tp;
    // tensor parallel: this exchange's sequence number (receive: the tag the
    // words must carry; send: the tag they get)
    const uint32_t tp_seq = TP && (tpa.tp_recv || tpa.tp_send) ? __ldcg(tp_ctl(tpa, tpa.tp_rank) + 2 + tpa.tp_par) + 1u : 0u;
    const unsigned long long tp_t0 = TP && tpa.tp_recv ? gtimer() : 0ull;
    bool tp_late = false;
    for (uint32_t base = 0; base < n4; base += T * NR) {
        float4 xv[NR];
        if (!TP || !tpa.tp_recv) {
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint32_t i = base + tid + T * r;
                xv[r] = i < n4 ? __ldcg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        } else {
            // the W received slots, added in rank order as the one-shot
            // all-reduce adds them
            tp_take_all<NR>(tpa, base, tid, T, n4, tp_seq, xv, tp_t0, tp_late);
        }
        if (a.x_copy && cta == 0 && !dry) {
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint32_t i = base + tid + T * r;
                if (i < n4) reinterpret_cast<float4*>(a.x_copy)[i] = xv[r];
            }
        }
        if (a.norm_w) {
            float4 gv[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint32_t i = base + tid + T * r;
                gv[r] = i < n4 ? g4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (base == 0) {
                // upstream rmsnorm.c: mean of squares, rsqrt + one Newton step
                // (the host only pairs a norm with K <= T*NR*4, one pass)
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
                for (uint32_t w = 0; w < NW; ++w) tot += rms_part[w];
                const float me = __fadd_rn(__fdiv_rn(tot, (float)a.K), a.eps);
                const float r0 = __fdiv_rn(1.0f, __fsqrt_rn(me));
                const float tm = __fsub_rn(3.0f, __fmul_rn(me, __fmul_rn(r0, r0)));
                r_norm = __fmul_rn(__fmul_rn(r0, tm), 0.5f);
            }
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                xv[r].x = __fmul_rn(__fmul_rn(xv[r].x, r_norm), gv[r].x);
                xv[r].y = __fmul_rn(__fmul_rn(xv[r].y, r_norm), gv[r].y);
                xv[r].z = __fmul_rn(__fmul_rn(xv[r].z, r_norm), gv[r].z);
                xv[r].w = __fmul_rn(__fmul_rn(xv[r].w, r_norm), gv[r].w);
            }
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const uint32_t i = base + tid + T * r;
            if (i < n4) {
                const uint32_t b = i / 8, q = i % 8;
                *reinterpret_cast<float4*>(bfrag + (size_t)b * GEMV_BFRAG_BYTES + q * 16) = xv[r];
            }
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(T));
    if (TP && tpa.tp_recv && tid == 0) tp_recv_done(tpa, tp_seq);
    for (uint32_t b = tid; b < nbk; b += T) {
        float v[32];
        const uint8_t* src = bfrag + (size_t)b * GEMV_BFRAG_BYTES;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 t4 = *reinterpret_cast<const float4*>(src + q * 16);
            v[4 * q] = t4.x;
            v[4 * q + 1] = t4.y;
            v[4 * q + 2] = t4.z;
            v[4 * q + 3] = t4.w;
        }
        float m = 0.0f;
#pragma unroll
        for (int k = 0; k < 32; ++k) m = fmaxf(m, fabsf(v[k]));
        // Grid 2^-sh with sh = 22 - e, m = f 2^e (f in [0.5, 1)): for a
        // normal m, e = E - 126 with E its biased exponent field.  A
        // subnormal m uses E = 1 (a coarser grid, still |X| <= 2^22), an
        // all-zero block any E.  v 2^sh is formed as two exact
        // power-of-two products (sh spans -106..147); an intermediate
        // can only lose bits when the final value rounds to 0 anyway.
        const int E = m > 0.0f ? max((int)(__float_as_uint(m) >> 23), 1) : 126;
        const int sh = 148 - E;
        int X[32];
        if (sh <= 127) {  // one exact product (every block but the tiniest)
            const float pw = __int_as_float((sh + 127) << 23);
#pragma unroll
            for (int k = 0; k < 32; ++k) X[k] = __float2int_rn(__fmul_rn(v[k], pw));
        } else {
            const int s1 = sh >> 1, s2 = sh - s1;
            const float p1 = __int_as_float((s1 + 127) << 23), p2 = __int_as_float((s2 + 127) << 23);
#pragma unroll
            for (int k = 0; k < 32; ++k) X[k] = __float2int_rn(__fmul_rn(__fmul_rn(v[k], p1), p2));
        }
        // Balanced limbs X = 65536 a + 256 b + c, b and c in [-128, 128):
        // c = X mod 256 (as a signed byte), b = floor((X + 128) / 256) mod
        // 256, a = floor((X + 32896) / 65536), i.e. byte 0 of X, byte 1 of
        // X + 0x80 and byte 2 of X + 0x8080; gathered four elements at a
        // time with byte permutes.  B fragment of lane L = g*4 + t (g < 3 =
        // limb): word 0 = limb g of k 4t..4t+3, word 1 = limb g of k
        // 16+4t..16+4t+3, so quad q (k = 4q..4q+3) is word 2*(q%4) + q/4 of
        // the limb's 32 bytes.
        uint32_t la[8], lb[8], lc[8];
        int sx = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint32_t x0 = (uint32_t)X[4 * q], x1 = (uint32_t)X[4 * q + 1];
            const uint32_t x2 = (uint32_t)X[4 * q + 2], x3 = (uint32_t)X[4 * q + 3];
            const int w = 2 * (q % 4) + q / 4;
            lc[w] = __byte_perm(__byte_perm(x0, x1, 0x0040), __byte_perm(x2, x3, 0x0040), 0x5410);
            lb[w] = __byte_perm(__byte_perm(x0 + 0x80u, x1 + 0x80u, 0x0051),
                                __byte_perm(x2 + 0x80u, x3 + 0x80u, 0x0051), 0x5410);
            la[w] = __byte_perm(__byte_perm(x0 + 0x8080u, x1 + 0x8080u, 0x0062),
                                __byte_perm(x2 + 0x8080u, x3 + 0x8080u, 0x0062), 0x5410);
            sx += (X[4 * q] + X[4 * q + 1]) + (X[4 * q + 2] + X[4 * q + 3]);
        }
        uint4* bf = reinterpret_cast<uint4*>(bfrag + (size_t)b * GEMV_BFRAG_BYTES);
        bf[0] = make_uint4(la[0], la[1], la[2], la[3]);
        bf[1] = make_uint4(la[4], la[5], la[6], la[7]);
        bf[2] = make_uint4(lb[0], lb[1], lb[2], lb[3]);
        bf[3] = make_uint4(lb[4], lb[5], lb[6], lb[7]);
        bf[4] = make_uint4(lc[0], lc[1], lc[2], lc[3]);
        bf[5] = make_uint4(lc[4], lc[5], lc[6], lc[7]);
        bf[6] = make_uint4(0u, 0u, 0u, 0u);  // column 3 (B lanes 12..15) is zero
        bf[7] = make_uint4(0u, 0u, 0u, 0u);
        // 2^-sh = 2^(E-148): normal for E >= 22, else the subnormal
        // 2^(E+1) * 2^-149.  Lane t of the D fragment: t = 0 weighs
        // 256*D_a + D_b by 256 f; t = 1 weighs D_c by f and adds the
        // -8*sum(X) correction; t = 2, 3 carry no limb and weigh 0.
        const float f = __uint_as_float(E >= 22 ? (uint32_t)(E - 21) << 23 : 1u << (E + 1));
        float4* fs = reinterpret_cast<float4*>(fsc + (size_t)b * 4);
        fs[0] = make_float4(f * 256.0f, 0.0f, f, f * (-8.0f * (float)sx));
        fs[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(T));
    if (dry) return;

    // ---- main loop ---------------------------------------------------------------
    const uint32_t g = lane >> 2, t = lane & 3;
    // D fragment of lane (g, t): rows g and g+8, columns 2t, 2t+1.  Columns
    // 0..2 are the limbs (a, b, c), column 3 is zero; B lanes 16..31 repeat
    // lanes 0..15, so columns 4..7 repeat 0..3 and lanes t >= 2 are
    // cancelled by zero weights.  p = D[2t] * m0 + D[2t+1]: t = 0 gives
    // 256*D_a + D_b, t = 1 gives D_c.
    const int m0 = t == 0 ? 256 : 1;
    const uint32_t ring_off = 0;
    const uint32_t bfrag_off = (uint32_t)(bfrag - smem) + (lane & 15) * 8;
    const uint32_t fsc_off = (uint32_t)(reinterpret_cast<uint8_t*>(fsc) - smem) + t * 8;
    // One block of a slab: bytes at smem + q (the lane's 16 weight bytes:
    // rows g, g+8 for the first mma, g+16, g+24 for the second), + sq (scales
    // of those four rows), + bq (limb fragment), + fq (grid factor,
    // correction).  Both mmas share the limb fragment.
    auto block_terms = [&](uint32_t q_off, uint32_t b_off, uint32_t f_off, float2& u01, float2& u23,
                           float4& sc) {
        const uint4 q = *reinterpret_cast<const uint4*>(smem + q_off);
        sc = *reinterpret_cast<const float4*>(smem + q_off + (512 + g * 16 - lane * 16));
        const uint2 bv = *reinterpret_cast<const uint2*>(smem + b_off);
        const float2 fz = *reinterpret_cast<const float2*>(smem + f_off);
        int d[4], e[4];
        mma_u8s8(d, q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, (q.x >> 4) & 0x0F0F0F0Fu,
                 (q.y >> 4) & 0x0F0F0F0Fu, bv.x, bv.y);
        mma_u8s8(e, q.z & 0x0F0F0F0Fu, q.w & 0x0F0F0F0Fu, (q.z >> 4) & 0x0F0F0F0Fu,
                 (q.w >> 4) & 0x0F0F0F0Fu, bv.x, bv.y);
        const float2 fw = make_float2(fz.x, fz.x), fc = make_float2(fz.y, fz.y);
        u01 = __ffma2_rn(make_float2((float)(d[0] * m0 + d[1]), (float)(d[2] * m0 + d[3])), fw, fc);
        u23 = __ffma2_rn(make_float2((float)(e[0] * m0 + e[1]), (float)(e[2] * m0 + e[3])), fw, fc);
    };
    // Slab sums wait in red[] (per warp) and are reduced by the whole CTA
    // every red_slabs slabs and at the end: warp w finishes slabs w, w+NW, ...
    // of the batch (cross-CTA parts through the ticket, then the epilogue).
    const uint32_t RS = c.red_slabs;
    uint32_t jl = 0, j_batch = j_first;
    auto reduce_batch = [&](uint32_t cnt) {
        asm volatile("bar.sync 1, %0;" ::"r"(T));
        for (uint32_t r = warp; r < cnt; r += NW) {
            const uint32_t j = j_batch + r;
            float v = 0.0f;
#pragma unroll
            for (uint32_t w = 0; w < NW; ++w) v += red[(r * NW + w) * GEMV_SLAB_ROWS + lane];
            const uint32_t c_first = j == j_first ? own_lo[0] : (j == j_last ? own_lo[1] : cta);
            const uint32_t c_last = j == j_first ? own_hi[0] : (j == j_last ? own_hi[1] : cta);
            bool finish = c_first == c_last;
            if (!finish) {
                float* pp = a.part + ((size_t)j * a.max_parts) * GEMV_SLAB_ROWS;
                pp[(cta - c_first) * GEMV_SLAB_ROWS + lane] = v;
                __syncwarp();
                // acq_rel ticket: releases this warp's parts, acquires the others'
                uint32_t last = 0;
                if (lane == 0) {
                    uint32_t old;
                    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                                 : "=r"(old)
                                 : "l"(&a.ticket[j])
                                 : "memory");
                    last = old == c_last - c_first ? 1u : 0u;
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    v = 0.0f;
                    for (uint32_t p = 0; p <= c_last - c_first; ++p) v += __ldcg(&pp[p * GEMV_SLAB_ROWS + lane]);
                    if (lane == 0) a.ticket[j] = 0u;
                    finish = true;
                }
            }
            if (finish) gemv_epilogue<TP>(a, c.tp, tp_seq, j, lane, v);
        }
        j_batch += cnt;
        jl = 0;
    };
    float2 acc = make_float2(0.0f, 0.0f), acc2 = make_float2(0.0f, 0.0f);  // rows g, g+8 | g+16, g+24
    // running ring slot / parity and current slab (no divisions per stage)
    uint32_t j = j_first, jb = j_first * nb;
    for (uint32_t sb0 = x0; sb0 < x1; sb0 += c.stage_blocks) {
        mbar_wait(&full[s], ph, QDEV_WAIT_FULL_TIMEOUT);
        const uint32_t sb1 = min(sb0 + c.stage_blocks, x1);
        for (uint32_t seg = sb0; seg < sb1;) {
            const uint32_t seg_end = min(sb1, jb + nb);
            // this warp's blocks of the segment: (b - jb) % NW == warp
            const uint32_t b = seg + ((warp + NW - (seg - jb) % NW) % NW);
            int n = b < seg_end ? (int)((seg_end - b + NW - 1) / NW) : 0;
            uint32_t qo = ring_off + s * stage_bytes + (b - sb0) * GEMV_BLOCK_BYTES + lane * 16;
            uint32_t bo = bfrag_off + (b - jb) * GEMV_BFRAG_BYTES;
            uint32_t fo = fsc_off + (b - jb) * GEMV_FSC_BYTES;
            constexpr uint32_t QS = NW * GEMV_BLOCK_BYTES, BS = NW * GEMV_BFRAG_BYTES, FS = NW * GEMV_FSC_BYTES;
            // four independent blocks per step, accumulated in block order
            for (; n >= 4; n -= 4, qo += 4 * QS, bo += 4 * BS, fo += 4 * FS) {
                float2 u01[4], u23[4];
                float4 sc[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    block_terms(qo + i * QS, bo + i * BS, fo + i * FS, u01[i], u23[i], sc[i]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc = __ffma2_rn(make_float2(sc[i].x, sc[i].y), u01[i], acc);
                    acc2 = __ffma2_rn(make_float2(sc[i].z, sc[i].w), u23[i], acc2);
                }
            }
            for (; n > 0; --n, qo += QS, bo += BS, fo += FS) {
                float2 u01, u23;
                float4 sc;
                block_terms(qo, bo, fo, u01, u23, sc);
                acc = __ffma2_rn(make_float2(sc.x, sc.y), u01, acc);
                acc2 = __ffma2_rn(make_float2(sc.z, sc.w), u23, acc2);
            }
            if (seg_end == jb + nb || seg_end == x1) {
                // slab j done for this warp: limbs (quad) -> red[jl][warp]
                float r4[4] = {acc.x, acc.y, acc2.x, acc2.y};  // rows g, g+8, g+16, g+24
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    r4[k] += __shfl_xor_sync(0xffffffffu, r4[k], 1);
                    r4[k] += __shfl_xor_sync(0xffffffffu, r4[k], 2);
                }
                if (t == 0) {
                    float* rr = red + (jl * NW + warp) * GEMV_SLAB_ROWS;
                    rr[g] = r4[0];
                    rr[g + 8] = r4[1];
                    rr[g + 16] = r4[2];
                    rr[g + 24] = r4[3];
                }
                acc = acc2 = make_float2(0.0f, 0.0f);
                if (++jl == RS) {
                    reduce_batch(RS);
                    asm volatile("bar.sync 1, %0;" ::"r"(T));  // red[] free again
                }
            }
            if (seg_end == jb + nb) {
                ++j;
                jb += nb;
            }
            seg = seg_end;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == c.n_stage) {
            s = 0;
            ph ^= 1;
        }
    }
    if (jl) reduce_batch(jl);
    asm volatile("bar.sync 1, %0;" ::"r"(T));  // tables and red[] free for the next phase
}

// TP: the single-phase tensor-parallel form (c.tp: exchange fused into
// the epilogue / prologue); the other instantiation carries none of it.
template <bool TP>
__global__ void __launch_bounds__(GEMV_THREADS, 1)
    q4_slab_kernel(const __grid_constant__ GemvChain c) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t NW = GEMV_CONSUMER_WARPS, T = NW * 32;
    const uint32_t stage_bytes = c.stage_blocks * GEMV_BLOCK_BYTES;
    uint8_t* ring = smem;
    uint8_t* bfrag = ring + (size_t)c.n_stage * stage_bytes;
    float2* fsc = reinterpret_cast<float2*>(bfrag + (size_t)c.max_nb * GEMV_BFRAG_BYTES);
    float* red = reinterpret_cast<float*>(fsc + (size_t)c.max_nb * 4);  // [red_slabs][NW][32]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)c.red_slabs * NW * GEMV_SLAB_ROWS);
    uint64_t* empty = full + 8;
    float* rms_part = reinterpret_cast<float*>(empty + 8);      // [NW]
    const uint32_t tid = threadIdx.x, G = gridDim.x, cta = blockIdx.x, P = c.n_phases;

    if (tid == 0) {
        for (uint32_t s = 0; s < c.n_stage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    // The phases' arguments, copied to shared memory before the dependency
    // wait: c.ph[p] with a run-time p is a generic load from the parameter
    // window, slow enough (about a microsecond per dependent chain) to show
    // on the critical path after the wait; shared-memory reads are not.
    __shared__ GemvArgs s_args[GEMV_MAX_PHASES];
    {
        static_assert(sizeof(GemvArgs) % 8 == 0, "GemvArgs copied as 64-bit words");
        constexpr uint32_t WORDS = sizeof(GemvArgs) / 8;
        const uint64_t* src = reinterpret_cast<const uint64_t*>(c.ph);
        uint64_t* dst = reinterpret_cast<uint64_t*>(s_args);
        for (uint32_t i = tid; i < P * WORDS; i += blockDim.x) dst[i] = src[i];
    }
    __shared__ PhaseRange s_rng[GEMV_MAX_PHASES];
    if (tid < P) s_rng[tid] = phase_range(c.ph[tid].n_slabs, c.ph[tid].nb, cta, G);
    __syncthreads();
    if (tid == 0) trace_mark(c.trace, 0);
    pdl_trigger();

    if (tid >= T) {
        // ---- producer warp: every phase's block range, back to back ----------
        if (tid == T) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t s = 0, ph = 0, k = 0;  // ring slot, its parity, stages issued
            bool ok = true;
            for (uint32_t p = 0; p < P && ok; ++p) {
                const GemvArgs& a = s_args[p];
                const uint32_t x0 = s_rng[p].x0, x1 = s_rng[p].x1;
                for (uint32_t b0 = x0; b0 < x1; b0 += c.stage_blocks, ++k) {
                    if (k >= c.n_stage && !mbar_wait(&empty[s], ph ^ 1, QDEV_WAIT_EMPTY_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    const uint32_t n = min(c.stage_blocks, x1 - b0);
                    mbar_arrive_expect_tx(&full[s], n * GEMV_BLOCK_BYTES);
                    bulk_g2s(ring + (size_t)s * stage_bytes, a.w + (size_t)b0 * GEMV_BLOCK_BYTES,
                             n * GEMV_BLOCK_BYTES, &full[s], pol);
                    if (++s == c.n_stage) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
        }
        pdl_wait();  // every thread waits: the grid ends after its predecessor
        return;
    }

    // ---- consumers -----------------------------------------------------------------
    uint32_t s = 0, ph = 0;
    // Iteration 0 would be a discarded ("dry") prologue pass before the
    // dependency wait; it measured slower, so the loop starts at 1.  The
    // loop keeps this shape because the simpler form compiled ~0.5% slower.
    constexpr uint32_t it0 = 1;
#pragma unroll 1
    for (uint32_t it = it0; it <= P; ++it) {
        const bool dry = it == 0;
        const uint32_t p = dry ? 0u : it - 1;
        if (it == 1) {
            pdl_wait();
            if (tid == 0) trace_mark(c.trace, 1);
        }
        if (p > 0) {
            // grid barrier: every CTA has finished phase p - 1 (outputs written)
            if (tid == 0) {
                const unsigned long long t0 = gtimer(), lim = qdev_wait_ns();
                while (ld_acquire_u32(c.bar + p - 1) < G) {
                    if (gtimer() - t0 > lim) {
                        qdev_fail(QDEV_GRID_TIMEOUT);
                        break;
                    }
                    __nanosleep(32);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(T));
        }
        gemv_phase<NW, TP>(s_args[p], c, smem, bfrag, fsc, red, full, empty, rms_part, s, ph, p, dry, s_rng[p]);
        if (dry) continue;
        if (p + 1 < P && tid == 0) {
            // consumers passed bar.sync at the end of the phase, so this
            // release covers every consumer thread's outputs
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(c.bar + p) : "memory");
        }
    }
    if (P > 1 && tid == 0) {
        // the last CTA out clears the counters for the next launch (all CTAs
        // are past every wait by then)
        __threadfence();
        if (atomicAdd(c.bar + P - 1, 1u) == G - 1) {
            for (uint32_t i = 0; i < P; ++i) c.bar[i] = 0u;
            __threadfence();
        }
    }
    if (tid == 0) trace_mark(c.trace, 2);
}

// Repack upstream AoS Q4_0 blocks ([M][nb] x 20 B) into slab tiles.
// interleave_half != 0: destination row 2i takes source row i and 2i+1 takes
// source row interleave_half + i (gate/up pairing).  Rows >= M are zero.
__global__ void q4_pack_kernel(const uint8_t* __restrict__ src, uint32_t M, uint32_t K,
                               uint32_t interleave_half, uint8_t* __restrict__ dst) {
    const uint32_t nb = K / 32;
    const uint32_t n_slabs = (M + GEMV_SLAB_ROWS - 1) / GEMV_SLAB_ROWS;
    const uint64_t n = (uint64_t)n_slabs * nb * 32;  // one thread per (slab, block, lane)
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t lane = (uint32_t)(i % 32);
        const uint64_t sb = i / 32;
        const uint32_t b = (uint32_t)(sb % nb), j = (uint32_t)(sb / nb);
        const uint32_t g = lane >> 2, t = lane & 3;
        uint8_t* out = dst + sb * GEMV_BLOCK_BYTES;
        uint32_t words[4];
        float scales[4];
        for (int quarter = 0; quarter < 4; ++quarter) {  // rows g, g+8, g+16, g+24
            const uint32_t drow = j * GEMV_SLAB_ROWS + g + 8 * quarter;
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
            words[quarter] = wv;
            scales[quarter] = sv;
        }
        *reinterpret_cast<uint4*>(out + lane * 16) = make_uint4(words[0], words[1], words[2], words[3]);
        if (t == 0)
            *reinterpret_cast<float4*>(out + 512 + g * 16) = make_float4(scales[0], scales[1], scales[2], scales[3]);
    }
}

}  // namespace qb200
