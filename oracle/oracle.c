/*
 * oracle.c — CPU restatement of the Qorus-IA forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker for the CUDA path.
 * Built with -std=c11 -ffp-contract=off so every a*b+c that upstream
 * writes unfused stays unfused; upstream's _mm256_fmadd_ps becomes fmaf.
 * Lane l of an upstream 8-wide accumulator is restated as element l of a
 * float[8], so the summation orders (and therefore the bits) match the
 * upstream AVX2 kernels.
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

typedef void (*rows_fn)(void* arg, uint32_t lo, uint32_t hi);
typedef struct { rows_fn fn; void* arg; uint32_t lo, hi; } rows_job;
static void* rows_thread(void* p) { rows_job* j = p; j->fn(j->arg, j->lo, j->hi); return NULL; }

static void par_rows(rows_fn fn, void* arg, uint32_t n) {
    int t = g_threads;
    if (t <= 1 || n < 64) { fn(arg, 0, n); return; }
    if ((uint32_t)t > n) t = (int)n;
    pthread_t th[256];
    rows_job jb[256];
    uint32_t chunk = (n + (uint32_t)t - 1) / (uint32_t)t;
    int k = 0;
    for (int i = 0; i < t; i++) {
        uint32_t lo = (uint32_t)i * chunk, hi = lo + chunk > n ? n : lo + chunk;
        if (lo >= hi) break;
        jb[k] = (rows_job){fn, arg, lo, hi};
        if (pthread_create(&th[k], NULL, rows_thread, &jb[k]) != 0) { fn(arg, lo, hi); continue; }
        k++;
    }
    for (int i = 0; i < k; i++) pthread_join(th[i], NULL);
}

/* The 4-lane tail of upstream horizontal_sum_avx / hsum256_ps
 * (avx_math.h:64-74, matmul_fp32.c:16-27): lanes l and l+4 are added, then
 * (s0+s1)+(s2+s3). */
static float hsum8(const float v[8]) {
    float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    return (s0 + s1) + (s2 + s3);
}

/* avx_math.h:10-61: degree-5 Taylor polynomial by Horner with FMA on x
 * clamped to [-5,5], floored at 0; x < -10 gives 0 and x > 10 gives 22026. */
float orc_exp_approx(float x) {
    if (x < -10.0f) return 0.0f;
    if (x > 10.0f) return 22026.0f;
    float c = x < 5.0f ? x : 5.0f;
    c = c > -5.0f ? c : -5.0f;
    float r = 0.00833333f;
    r = fmaf(r, c, 0.04166667f);
    r = fmaf(r, c, 0.16666667f);
    r = fmaf(r, c, 0.5f);
    r = fmaf(r, c, 1.0f);
    r = fmaf(r, c, 1.0f);
    return r > 0.0f ? r : 0.0f;
}

/* dequantize.c:18-73 and matmul.c:43-96: w = fma(q, s, -8*s), byte b giving
 * elements 2b (low nibble) and 2b+1 (high nibble). */
static inline void deq_block(const uint8_t* blk, float* w) {
    float s;
    memcpy(&s, blk + 16, 4);
    float off = -8.0f * s;
    for (int b = 0; b < 16; b++) {
        w[2 * b] = fmaf((float)(blk[b] & 15), s, off);
        w[2 * b + 1] = fmaf((float)(blk[b] >> 4), s, off);
    }
}

void orc_dequantize_block(const uint8_t* block20, float* out32) { deq_block(block20, out32); }

typedef struct { const uint8_t* w; uint32_t K; const float* x; float* y; } gemvq_job;

/* matmul.c:98-271: per row, block b feeds accumulator b % 4; inside a block
 * batch t (elements 8t..8t+7) accumulates lane-wise in order t = 0..3;
 * then (acc0+acc1)+(acc2+acc3) and the horizontal sum. */
static void gemvq_rows(void* a, uint32_t lo, uint32_t hi) {
    gemvq_job* j = a;
    uint32_t nb = j->K / 32;
    for (uint32_t r = lo; r < hi; r++) {
        float acc[4][8] = {{0}};
        const uint8_t* row = j->w + (size_t)r * nb * 20;
        for (uint32_t b = 0; b < nb; b++) {
            float w[32];
            deq_block(row + (size_t)b * 20, w);
            const float* xb = j->x + (size_t)b * 32;
            float* A = acc[b & 3];
            for (int t = 0; t < 4; t++)
                for (int l = 0; l < 8; l++) A[l] = fmaf(w[8 * t + l], xb[8 * t + l], A[l]);
        }
        float v[8];
        for (int l = 0; l < 8; l++) v[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
        j->y[r] = hsum8(v);
    }
}

int orc_gemv_q4(const uint8_t* w, uint32_t M, uint32_t K, const float* x, float* y) {
    if (!w || !x || !y) return -10;
    if (M == 0 || K == 0 || K % 32) return -15;
    gemvq_job j = {w, K, x, y};
    par_rows(gemvq_rows, &j, M);
    return 0;
}

/* matmul_fp32.c:388-471. */
float orc_dot_f32(const float* a, const float* b, uint32_t K) {
    uint32_t kv = K & ~31u;
    float dot = 0.0f;
    if (kv) {
        float acc[4][8] = {{0}};
        for (uint32_t k = 0; k < kv; k += 32)
            for (int q = 0; q < 4; q++)
                for (int l = 0; l < 8; l++)
                    acc[q][l] = fmaf(a[k + 8 * q + l], b[k + 8 * q + l], acc[q][l]);
        float v[8];
        for (int l = 0; l < 8; l++) v[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
        dot = hsum8(v);
    }
    for (uint32_t k = kv; k < K; k++) {
        float p = a[k] * b[k];
        dot = dot + p;
    }
    return dot;
}

typedef struct { const float* w; uint32_t K; const float* x; float* y; } gemvf_job;
static void gemvf_rows(void* a, uint32_t lo, uint32_t hi) {
    gemvf_job* j = a;
    for (uint32_t r = lo; r < hi; r++) j->y[r] = orc_dot_f32(j->w + (size_t)r * j->K, j->x, j->K);
}

int orc_gemv_f32(const float* w, uint32_t M, uint32_t K, const float* x, float* y) {
    if (!w || !x || !y) return -10;
    if (M == 0 || K == 0) return -15;
    gemvf_job j = {w, K, x, y};
    par_rows(gemvf_rows, &j, M);
    return 0;
}

/* rmsnorm.c:15-92. */
int orc_rmsnorm(const float* x, const float* w, float* out, uint32_t N, float eps) {
    if (!x || !w || !out) return -10;
    if (N == 0 || N % 8) return -15;
    float acc[8] = {0};
    for (uint32_t i = 0; i < N; i += 8)
        for (int l = 0; l < 8; l++) {
            float sq = x[i + l] * x[i + l];
            acc[l] = acc[l] + sq;
        }
    float sum = hsum8(acc);
    float mean = sum / (float)N;
    float me = mean + eps;
    float r0 = 1.0f / sqrtf(me);
    float rsq = r0 * r0;
    float xr = me * rsq;
    float tm = 3.0f - xr;
    float r = (r0 * tm) * 0.5f;
    for (uint32_t i = 0; i < N; i++) {
        float n = x[i] * r;
        out[i] = n * w[i];
    }
    return 0;
}

/* rope.c:23-110: even lane x*c - y*s, odd lane y*c + x*s (addsub of two
 * unfused products). */
int orc_rope(const float* x, const float* c, const float* s, float* out, uint32_t N) {
    if (!x || !c || !s || !out) return -10;
    if (N == 0 || N % 8) return -15;
    for (uint32_t i = 0; i < N; i += 2) {
        float t0 = x[i] * c[i], t1 = x[i + 1] * c[i + 1];
        float u0 = x[i + 1] * s[i], u1 = x[i] * s[i + 1];
        out[i] = t0 - u0;
        out[i + 1] = t1 + u1;
    }
    return 0;
}

/* softmax.c:17-132. */
int orc_softmax(const float* x, float* out, uint32_t N) {
    if (!x || !out) return -10;
    if (N == 0) return -15;
    if (N < 8) {
        float m = x[0];
        for (uint32_t i = 1; i < N; i++)
            if (x[i] > m) m = x[i];
        float sum = 0.0f;
        for (uint32_t i = 0; i < N; i++) {
            float e = expf(x[i] - m);
            out[i] = e;
            sum += e;
        }
        for (uint32_t i = 0; i < N; i++) out[i] /= sum;
        return 0;
    }
    uint32_t nv = N / 8 * 8;
    float m = -INFINITY;
    for (uint32_t i = 0; i < nv; i++)
        if (x[i] > m) m = x[i];
    for (uint32_t i = nv; i < N; i++)
        if (x[i] > m) m = x[i];
    float acc[8] = {0};
    for (uint32_t i = 0; i < nv; i += 8)
        for (int l = 0; l < 8; l++) {
            float e = orc_exp_approx(x[i + l] - m);
            acc[l] = acc[l] + e;
            out[i + l] = e;
        }
    float sum = hsum8(acc);
    for (uint32_t i = nv; i < N; i++) {
        float e = expf(x[i] - m);
        out[i] = e;
        sum += e;
    }
    float inv = 1.0f / sum;
    for (uint32_t i = 0; i < N; i++) out[i] = out[i] * inv;
    return 0;
}

/* silu.c:18-94. */
int orc_silu(const float* x, float* out, uint32_t N) {
    if (!x || !out) return -10;
    if (N == 0) return -15;
    uint32_t nv = N < 8 ? 0 : N / 8 * 8;
    for (uint32_t i = 0; i < nv; i++) {
        float e = orc_exp_approx(-x[i]);
        float d = 1.0f + e;
        float sg = 1.0f / d;
        out[i] = x[i] * sg;
    }
    for (uint32_t i = nv; i < N; i++) {
        float sg = 1.0f / (1.0f + expf(-x[i]));
        out[i] = x[i] * sg;
    }
    return 0;
}

/* model.c:625-665. */
void orc_rope_tables(float theta, uint32_t hd, uint32_t max_seq, float* ct, float* st) {
    uint32_t np = hd / 2;
    float* fr = malloc(sizeof(float) * (np ? np : 1));
    for (uint32_t i = 0; i < np; i++) {
        float e = -2.0f * (float)i / (float)hd;
        fr[i] = powf(theta, e);
    }
    for (uint32_t p = 0; p < max_seq; p++)
        for (uint32_t i = 0; i < np; i++) {
            float th = fr[i] * (float)p;
            float c = cosf(th), s = sinf(th);
            size_t o = (size_t)p * hd + (size_t)i * 2;
            ct[o] = ct[o + 1] = c;
            st[o] = st[o + 1] = s;
        }
    free(fr);
}

uint32_t orc_argmax(const float* x, uint32_t n) {
    uint32_t bi = 0;
    float bv = x[0];
    for (uint32_t i = 1; i < n; i++)
        if (x[i] > bv) { bv = x[i]; bi = i; }
    return bi;
}

/* ---- model ------------------------------------------------------------- */

static size_t al64(size_t n) { return (n + 63) & ~(size_t)63; }

int orc_model_open(orc_model* m, const void* file, size_t size) {
    if (!m || !file) return -1;
    memset(m, 0, sizeof *m);
    if (size < 64) return -4;
    const uint32_t* h = file;
    if (h[0] != 0x514F5231u) return -6;
    m->vocab = h[2]; m->dim = h[3]; m->hidden = h[4]; m->n_layers = h[5];
    m->n_heads = h[6]; m->n_kv_heads = h[7]; m->max_seq = h[8];
    memcpy(&m->theta, h + 9, 4);
    float eps;
    memcpy(&eps, h + 10, 4);
    m->eps = (h[1] >= 2 && eps > 0.0f) ? eps : 1e-5f; /* model.c:339-343 */
    if (!m->vocab || !m->dim || !m->n_layers || !m->n_heads || !m->n_kv_heads) return -9;
    if (m->dim % 32 || m->hidden % 32 || m->n_layers > 512) return -9;
    size_t D = m->dim, H = m->hidden, V = m->vocab, hd = D / m->n_heads;
    size_t kvd = m->n_kv_heads * hd;
    const uint8_t* base = file;
    size_t off = 64;
#define TAKE(dst, T, bytes)                     \
    do {                                        \
        if (off + (bytes) > size) return -9;    \
        dst = (const T*)(base + off);           \
        off += al64(bytes);                     \
    } while (0)
    TAKE(m->token_embd, float, V * D * 4);
    TAKE(m->output_norm, float, D * 4);
    TAKE(m->output, float, V * D * 4);
    for (uint32_t l = 0; l < m->n_layers; l++) {
        TAKE(m->attn_norm[l], float, D * 4);
        TAKE(m->wq[l], uint8_t, D * (D / 32) * 20);
        TAKE(m->wk[l], uint8_t, kvd * (D / 32) * 20);
        TAKE(m->wv[l], uint8_t, kvd * (D / 32) * 20);
        TAKE(m->wo[l], uint8_t, D * (D / 32) * 20);
        TAKE(m->ffn_norm[l], float, D * 4);
        TAKE(m->w_gate[l], uint8_t, H * (D / 32) * 20);
        TAKE(m->w_up[l], uint8_t, H * (D / 32) * 20);
        TAKE(m->w_down[l], uint8_t, D * (H / 32) * 20);
    }
#undef TAKE
    m->cos_tab = malloc((size_t)m->max_seq * hd * sizeof(float) + 64);
    m->sin_tab = malloc((size_t)m->max_seq * hd * sizeof(float) + 64);
    if (!m->cos_tab || !m->sin_tab) return -7;
    orc_rope_tables(m->theta, (uint32_t)hd, m->max_seq, m->cos_tab, m->sin_tab);
    return 0;
}

void orc_model_close(orc_model* m) {
    if (!m) return;
    free(m->cos_tab);
    free(m->sin_tab);
    m->cos_tab = m->sin_tab = NULL;
}

typedef struct {
    const orc_model* m;
    const float* kv;
    const float* q;   /* [S][D] rotated */
    float* att;       /* [S][D] */
    uint32_t S, pos, T, hd;
    size_t head_stride, layer_base;
} attn_job;

/* model.c:1226-1438 restated over the cache: per (row t, head qh) the
 * scores q.k_j (matmul_fp32 dot order) times 1/sqrt(hd), the causal mask
 * -1e9 for j > pos+t, softmax over the full row of T = pos+S entries, then
 * out[d] = dot(P, V[:, d]) in the same dot order. */
static void attn_rows(void* a, uint32_t lo, uint32_t hi) {
    attn_job* j = a;
    const orc_model* m = j->m;
    uint32_t hd = j->hd, T = j->T, D = m->dim;
    uint32_t group = m->n_heads / m->n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    float* sc = malloc(sizeof(float) * T);
    float* pr = malloc(sizeof(float) * T);
    float* vc = malloc(sizeof(float) * T);
    for (uint32_t item = lo; item < hi; item++) {
        uint32_t t = item / m->n_heads, qh = item % m->n_heads;
        uint32_t kvh = qh / group;
        const float* slab = j->kv + j->layer_base + (size_t)kvh * j->head_stride;
        const float* qv = j->q + (size_t)t * D + (size_t)qh * hd;
        uint32_t last = j->pos + t;
        for (uint32_t p = 0; p < T; p++) {
            if (p > last) { sc[p] = -1e9f; continue; }
            float d = orc_dot_f32(qv, slab + (size_t)p * 2 * hd, hd);
            sc[p] = d * scale;
        }
        orc_softmax(sc, pr, T);
        float* o = j->att + (size_t)t * D + (size_t)qh * hd;
        for (uint32_t d = 0; d < hd; d++) {
            for (uint32_t p = 0; p < T; p++) vc[p] = slab[(size_t)p * 2 * hd + hd + d];
            o[d] = orc_dot_f32(pr, vc, T);
        }
    }
    free(sc);
    free(pr);
    free(vc);
}

int orc_forward(const orc_model* m, float* kv, const uint32_t* tokens, uint32_t S,
                uint32_t pos, float* logits) {
    if (!m || !kv || !tokens || !logits) return -10;
    if (S == 0 || S > m->max_seq) return -15;
    if (pos >= m->max_seq || pos + S > m->max_seq) return -10;
    uint32_t D = m->dim, H = m->hidden, hd = D / m->n_heads;
    uint32_t kvd = m->n_kv_heads * hd;
    size_t SD = (size_t)S * D;
    float* x = malloc(SD * 4);
    float* xn = malloc(SD * 4);
    float* q = malloc(SD * 4);
    float* qr = malloc(SD * 4);
    float* k = malloc((size_t)S * kvd * 4);
    float* v = malloc((size_t)S * kvd * 4);
    float* att = malloc(SD * 4);
    float* ao = malloc(SD * 4);
    float* g = malloc((size_t)S * H * 4);
    float* u = malloc((size_t)S * H * 4);
    float* gs = malloc((size_t)S * H * 4);
    float* mo = malloc(SD * 4);
    float* tmp = malloc((size_t)hd * 4);
    int rc = 0;
    if (!x || !xn || !q || !qr || !k || !v || !att || !ao || !g || !u || !gs || !mo || !tmp) {
        rc = -7;
        goto out;
    }
    /* model.c:1027-1068 */
    for (uint32_t t = 0; t < S; t++) {
        if (tokens[t] >= m->vocab) { rc = -10; goto out; }
        memcpy(x + (size_t)t * D, m->token_embd + (size_t)tokens[t] * D, (size_t)D * 4);
    }
    size_t head_stride = (size_t)m->max_seq * 2 * hd;
    size_t layer_stride = head_stride * m->n_kv_heads;
    for (uint32_t l = 0; l < m->n_layers; l++) {
        for (uint32_t t = 0; t < S; t++)
            orc_rmsnorm(x + (size_t)t * D, m->attn_norm[l], xn + (size_t)t * D, D, m->eps);
        for (uint32_t t = 0; t < S; t++) {
            orc_gemv_q4(m->wq[l], D, D, xn + (size_t)t * D, q + (size_t)t * D);
            orc_gemv_q4(m->wk[l], kvd, D, xn + (size_t)t * D, k + (size_t)t * kvd);
            orc_gemv_q4(m->wv[l], kvd, D, xn + (size_t)t * D, v + (size_t)t * kvd);
        }
        /* model.c:1170-1222: rotate q and k heads, store K|V at pos+t */
        for (uint32_t t = 0; t < S; t++) {
            const float* ct = m->cos_tab + (size_t)(pos + t) * hd;
            const float* st = m->sin_tab + (size_t)(pos + t) * hd;
            for (uint32_t h = 0; h < m->n_heads; h++)
                orc_rope(q + (size_t)t * D + h * hd, ct, st, qr + (size_t)t * D + h * hd, hd);
            for (uint32_t h = 0; h < m->n_kv_heads; h++) {
                float* dst = kv + (size_t)l * layer_stride + h * head_stride +
                             (size_t)(pos + t) * 2 * hd;
                orc_rope(k + (size_t)t * kvd + h * hd, ct, st, tmp, hd);
                memcpy(dst, tmp, (size_t)hd * 4);
                memcpy(dst + hd, v + (size_t)t * kvd + h * hd, (size_t)hd * 4);
            }
        }
        attn_job aj = {m, kv, qr, att, S, pos, pos + S, hd, head_stride, (size_t)l * layer_stride};
        par_rows(attn_rows, &aj, S * m->n_heads);
        for (uint32_t t = 0; t < S; t++)
            orc_gemv_q4(m->wo[l], D, D, att + (size_t)t * D, ao + (size_t)t * D);
        /* model.c:1620-1647: x1 = x + attn; mlp on rmsnorm(x1); x = x1 + mlp */
        for (size_t i = 0; i < SD; i++) x[i] = x[i] + ao[i];
        for (uint32_t t = 0; t < S; t++)
            orc_rmsnorm(x + (size_t)t * D, m->ffn_norm[l], xn + (size_t)t * D, D, m->eps);
        for (uint32_t t = 0; t < S; t++) {
            orc_gemv_q4(m->w_gate[l], H, D, xn + (size_t)t * D, g + (size_t)t * H);
            orc_gemv_q4(m->w_up[l], H, D, xn + (size_t)t * D, u + (size_t)t * H);
        }
        /* model.c:1516-1549: silu over the whole [S*H] buffer, then mul */
        orc_silu(g, gs, S * H);
        for (size_t i = 0; i < (size_t)S * H; i++) gs[i] = gs[i] * u[i];
        for (uint32_t t = 0; t < S; t++)
            orc_gemv_q4(m->w_down[l], D, H, gs + (size_t)t * H, mo + (size_t)t * D);
        for (size_t i = 0; i < SD; i++) x[i] = x[i] + mo[i];
    }
    /* model.c:1799-1844: final norm of the last row, FP32 LM head */
    orc_rmsnorm(x + (size_t)(S - 1) * D, m->output_norm, xn, D, m->eps);
    orc_gemv_f32(m->output, m->vocab, D, xn, logits);
out:
    free(x); free(xn); free(q); free(qr); free(k); free(v); free(att); free(ao);
    free(g); free(u); free(gs); free(mo); free(tmp);
    return rc;
}
