/*
 * ref_forward.c — the intended Llama-3 forward composed from the UPSTREAM
 * AVX2 kernels themselves (q_gemv_q4_f32_avx2, q_rmsnorm_f32_avx2,
 * q_rope_f32_avx2, q_matmul_f32_avx2, q_softmax_f32_avx2, q_silu_f32_avx2,
 * q_mul_f32_avx2, q_add_f32_avx2), linked from oracle/_ref/libqorus_ref.so
 * which oracle/Makefile compiles from the upstream sources in place.
 *
 * TEST INFRASTRUCTURE ONLY.  Two uses: (1) it pins the C restatement in
 * oracle.c against the real upstream kernels on whole forwards; (2) it is
 * bench.py's `--impl reference` arm, the upstream CPU implementation of the
 * path timed on the host.  Upstream is single-threaded; rf_set_threads(n)
 * splits independent rows / heads over n host threads, each thread calling
 * the unmodified upstream kernels on its slice (results are identical for
 * any n because every output element is computed by one kernel call).
 *
 * Graph: the one upstream src/models/model.c:1088-1850 intends — [out][in]
 * weights, RMSNorm per row, attention over cache positions 0..pos+t with
 * GQA (kv head = qh / (n_heads / n_kv_heads), model.c:1311).
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "qorus.h" /* the upstream header, from the upstream include dir */

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    uint32_t vocab, dim, hidden, n_layers, n_heads, n_kv_heads, max_seq;
    float theta, eps;
    const float* token_embd;
    const float* output_norm;
    const float* output;
    const float** attn_norm;
    const q_block_q4_0** wq;
    const q_block_q4_0** wk;
    const q_block_q4_0** wv;
    const q_block_q4_0** wo;
    const float** ffn_norm;
    const q_block_q4_0** w_gate;
    const q_block_q4_0** w_up;
    const q_block_q4_0** w_down;
    float* cos_tab;
    float* sin_tab;
} rf_model;

static int g_nt = 1;
void rf_set_threads(int n) { g_nt = n < 1 ? 1 : (n > 256 ? 256 : n); }

static size_t al64(size_t n) { return (n + 63) & ~(size_t)63; }

static void* xalloc(size_t n) {
    void* p = NULL;
    if (posix_memalign(&p, 64, al64(n ? n : 64)) != 0) return NULL;
    return p;
}

void rf_close(void* h) {
    rf_model* m = h;
    if (!m) return;
    free(m->attn_norm); free(m->wq); free(m->wk); free(m->wv); free(m->wo);
    free(m->ffn_norm); free(m->w_gate); free(m->w_up); free(m->w_down);
    free(m->cos_tab); free(m->sin_tab);
    free(m);
}

void* rf_open(const void* file, size_t size) {
    const uint32_t* h = file;
    if (!file || size < 64 || h[0] != Q_MAGIC) return NULL;
    rf_model* m = calloc(1, sizeof *m);
    m->vocab = h[2]; m->dim = h[3]; m->hidden = h[4]; m->n_layers = h[5];
    m->n_heads = h[6]; m->n_kv_heads = h[7]; m->max_seq = h[8];
    memcpy(&m->theta, h + 9, 4);
    float eps;
    memcpy(&eps, h + 10, 4);
    m->eps = (h[1] >= 2 && eps > 0.0f) ? eps : 1e-5f;
    uint32_t L = m->n_layers;
    m->attn_norm = calloc(L, sizeof(void*)); m->ffn_norm = calloc(L, sizeof(void*));
    m->wq = calloc(L, sizeof(void*)); m->wk = calloc(L, sizeof(void*));
    m->wv = calloc(L, sizeof(void*)); m->wo = calloc(L, sizeof(void*));
    m->w_gate = calloc(L, sizeof(void*)); m->w_up = calloc(L, sizeof(void*));
    m->w_down = calloc(L, sizeof(void*));
    size_t D = m->dim, H = m->hidden, V = m->vocab, hd = D / m->n_heads;
    size_t kvd = m->n_kv_heads * hd, off = 64;
    const uint8_t* b = file;
#define TAKE(dst, T, bytes) do { if (off + (bytes) > size) { rf_close(m); return NULL; } \
        dst = (const T*)(b + off); off += al64(bytes); } while (0)
    TAKE(m->token_embd, float, V * D * 4);
    TAKE(m->output_norm, float, D * 4);
    TAKE(m->output, float, V * D * 4);
    for (uint32_t l = 0; l < L; l++) {
        TAKE(m->attn_norm[l], float, D * 4);
        TAKE(m->wq[l], q_block_q4_0, D * (D / 32) * 20);
        TAKE(m->wk[l], q_block_q4_0, kvd * (D / 32) * 20);
        TAKE(m->wv[l], q_block_q4_0, kvd * (D / 32) * 20);
        TAKE(m->wo[l], q_block_q4_0, D * (D / 32) * 20);
        TAKE(m->ffn_norm[l], float, D * 4);
        TAKE(m->w_gate[l], q_block_q4_0, H * (D / 32) * 20);
        TAKE(m->w_up[l], q_block_q4_0, H * (D / 32) * 20);
        TAKE(m->w_down[l], q_block_q4_0, D * (H / 32) * 20);
    }
#undef TAKE
    /* model.c:625-665 */
    size_t np = hd / 2;
    m->cos_tab = xalloc((size_t)m->max_seq * hd * 4);
    m->sin_tab = xalloc((size_t)m->max_seq * hd * 4);
    float* fr = malloc(np * 4 + 4);
    for (size_t i = 0; i < np; i++) fr[i] = powf(m->theta, -2.0f * (float)i / (float)hd);
    for (size_t p = 0; p < m->max_seq; p++)
        for (size_t i = 0; i < np; i++) {
            float th = fr[i] * (float)p;
            float c = cosf(th), s = sinf(th);
            m->cos_tab[p * hd + 2 * i] = m->cos_tab[p * hd + 2 * i + 1] = c;
            m->sin_tab[p * hd + 2 * i] = m->sin_tab[p * hd + 2 * i + 1] = s;
        }
    free(fr);
    return m;
}

/* ---- row-parallel helpers over the upstream kernels -------------------- */

typedef struct {
    int kind; /* 0 q4 gemv, 1 f32 head */
    const void* w;
    uint32_t K;
    const float* x;
    float* y;
    uint32_t lo, hi;
    int rc;
} gemv_part;

static void* gemv_worker(void* p) {
    gemv_part* g = p;
    uint32_t rows = g->hi - g->lo;
    if (g->kind == 0) {
        q_tensor w;
        memset(&w, 0, sizeof w);
        w.data = (void*)((const q_block_q4_0*)g->w + (size_t)g->lo * (g->K / 32));
        w.ne[0] = rows; w.ne[1] = g->K; w.ne[2] = w.ne[3] = 1;
        w.nb[0] = (size_t)(g->K / 32) * sizeof(q_block_q4_0);
        w.nb[1] = w.nb[2] = w.nb[3] = sizeof(q_block_q4_0);
        w.type = Q_Q4_0;
        /* upstream requires a 32-byte aligned output: use a private buffer */
        float* y = xalloc((size_t)rows * 4);
        g->rc = q_gemv_q4_f32_avx2(&w, g->x, y);
        memcpy(g->y + g->lo, y, (size_t)rows * 4);
        free(y);
    } else {
        /* model.c:1821-1844: last_token [1,D] @ transposed output view [D,V] */
        q_context c;
        memset(&c, 0, sizeof c);
        q_alloc_arena(&c, 1 << 16);
        q_tensor a, b, o;
        memset(&a, 0, sizeof a); memset(&b, 0, sizeof b); memset(&o, 0, sizeof o);
        a.data = (void*)g->x; a.ne[0] = 1; a.ne[1] = g->K; a.ne[2] = a.ne[3] = 1;
        a.nb[0] = (size_t)g->K * 4; a.nb[1] = a.nb[2] = a.nb[3] = 4; a.type = Q_F32;
        b.data = (void*)((const float*)g->w + (size_t)g->lo * g->K);
        b.ne[0] = g->K; b.ne[1] = rows; b.ne[2] = b.ne[3] = 1;
        b.nb[0] = 4; b.nb[1] = (size_t)g->K * 4; b.nb[2] = b.nb[3] = 4; b.type = Q_F32;
        float* y = xalloc((size_t)rows * 4);
        o.data = y; o.ne[0] = 1; o.ne[1] = rows; o.ne[2] = o.ne[3] = 1;
        o.nb[0] = (size_t)rows * 4; o.nb[1] = o.nb[2] = o.nb[3] = 4; o.type = Q_F32;
        g->rc = q_matmul_f32_avx2(&a, &b, &o, &c);
        memcpy(g->y + g->lo, y, (size_t)rows * 4);
        free(y);
        q_free_memory(&c);
    }
    return NULL;
}

static int par_gemv(int kind, const void* w, uint32_t M, uint32_t K, const float* x, float* y) {
    int nt = g_nt;
    if ((uint32_t)nt > M / 8) nt = M / 8 ? (int)(M / 8) : 1;
    gemv_part parts[256];
    pthread_t th[256];
    uint32_t chunk = (M + (uint32_t)nt - 1) / (uint32_t)nt;
    int n = 0;
    for (int i = 0; i < nt; i++) {
        uint32_t lo = (uint32_t)i * chunk, hi = lo + chunk > M ? M : lo + chunk;
        if (lo >= hi) break;
        parts[n] = (gemv_part){kind, w, K, x, y, lo, hi, 0};
        n++;
    }
    for (int i = 1; i < n; i++) pthread_create(&th[i], NULL, gemv_worker, &parts[i]);
    gemv_worker(&parts[0]);
    for (int i = 1; i < n; i++) pthread_join(th[i], NULL);
    for (int i = 0; i < n; i++)
        if (parts[i].rc) return parts[i].rc;
    return 0;
}

typedef struct {
    const rf_model* m;
    const float* kv;
    const float* q;
    float* att;
    uint32_t S, pos, T, hd;
    size_t head_stride, layer_base;
    uint32_t lo, hi;
    int rc;
} attn_part;

/* model.c:1226-1438 over the cache, one (row, head) item at a time. */
static void* attn_worker(void* p) {
    attn_part* j = p;
    const rf_model* m = j->m;
    uint32_t hd = j->hd, T = j->T, D = m->dim, group = m->n_heads / m->n_kv_heads;
    size_t rowb = al64((size_t)T * 4);
    float scale = 1.0f / sqrtf((float)hd);
    float* sc = xalloc(rowb);
    float* qv = xalloc((size_t)hd * 4);
    float* o = xalloc((size_t)hd * 4);
    float* kd = xalloc((size_t)T * hd * 4);
    q_context c;
    memset(&c, 0, sizeof c);
    q_alloc_arena(&c, al64((size_t)T * hd * 4) + 4096);
    for (uint32_t item = j->lo; item < j->hi; item++) {
        uint32_t t = item / m->n_heads, qh = item % m->n_heads, kvh = qh / group;
        const float* slab = j->kv + j->layer_base + (size_t)kvh * j->head_stride;
        memcpy(qv, j->q + (size_t)t * D + (size_t)qh * hd, (size_t)hd * 4);
        q_tensor a, b, o_t;
        memset(&a, 0, sizeof a); memset(&b, 0, sizeof b); memset(&o_t, 0, sizeof o_t);
        /* scores [1,T] = q [1,hd] @ K^T as a transposed [hd,T] view */
        a.data = qv; a.ne[0] = 1; a.ne[1] = hd; a.ne[2] = a.ne[3] = 1;
        a.nb[0] = (size_t)hd * 4; a.nb[1] = a.nb[2] = a.nb[3] = 4; a.type = Q_F32;
        /* the upstream transposed-B path strides columns by K (matmul_fp32.c
         * B_T_col = B_T_data + jj*K), so the K rows are gathered densely first,
         * as upstream's own k_heads buffer is (model.c:1237-1245) */
        for (uint32_t p2 = 0; p2 < T; p2++)
            memcpy(kd + (size_t)p2 * hd, slab + (size_t)p2 * 2 * hd, (size_t)hd * 4);
        b.data = kd; b.ne[0] = hd; b.ne[1] = T; b.ne[2] = b.ne[3] = 1;
        b.nb[0] = 4; b.nb[1] = (size_t)hd * 4; b.nb[2] = b.nb[3] = 4; b.type = Q_F32;
        o_t.data = sc; o_t.ne[0] = 1; o_t.ne[1] = T; o_t.ne[2] = o_t.ne[3] = 1;
        o_t.nb[0] = rowb; o_t.nb[1] = o_t.nb[2] = o_t.nb[3] = 4; o_t.type = Q_F32;
        int rc = q_matmul_f32_avx2(&a, &b, &o_t, &c);
        q_arena_reset(&c);
        if (rc) { j->rc = rc; break; }
        uint32_t last = j->pos + t;
        for (uint32_t p2 = 0; p2 < T; p2++) sc[p2] *= scale;   /* model.c:1376 */
        for (uint32_t p2 = last + 1; p2 < T; p2++) sc[p2] = -1e9f; /* causal mask */
        rc = q_softmax_f32_avx2(sc, sc, T);
        if (rc) { j->rc = rc; break; }
        /* out [1,hd] = P [1,T] @ V [T,hd] (row stride 2*hd: upstream transposes B) */
        a.data = sc; a.ne[1] = T; a.nb[0] = rowb;
        b.data = (void*)(slab + hd); b.ne[0] = T; b.ne[1] = hd;
        b.nb[0] = (size_t)2 * hd * 4; b.nb[1] = 4;
        o_t.data = o; o_t.ne[1] = hd; o_t.nb[0] = (size_t)hd * 4;
        rc = q_matmul_f32_avx2(&a, &b, &o_t, &c);
        q_arena_reset(&c);
        if (rc) { j->rc = rc; break; }
        memcpy(j->att + (size_t)t * D + (size_t)qh * hd, o, (size_t)hd * 4);
    }
    q_free_memory(&c);
    free(sc); free(qv); free(o); free(kd);
    return NULL;
}

static int vec_op(int mul, float* a, const float* b, float* out, size_t n) {
    q_tensor ta, tb, to;
    memset(&ta, 0, sizeof ta); memset(&tb, 0, sizeof tb); memset(&to, 0, sizeof to);
    ta.data = a; tb.data = (void*)b; to.data = out;
    ta.ne[0] = tb.ne[0] = to.ne[0] = (uint32_t)n;
    ta.ne[1] = tb.ne[1] = to.ne[1] = ta.ne[2] = tb.ne[2] = to.ne[2] = 1;
    ta.ne[3] = tb.ne[3] = to.ne[3] = 1;
    ta.nb[0] = tb.nb[0] = to.nb[0] = n * 4;
    ta.nb[1] = tb.nb[1] = to.nb[1] = 4; ta.nb[2] = tb.nb[2] = to.nb[2] = 4;
    ta.nb[3] = tb.nb[3] = to.nb[3] = 4;
    ta.type = tb.type = to.type = Q_F32;
    return mul ? q_mul_f32_avx2(&ta, &tb, &to) : q_add_f32_avx2(&ta, &tb, &to);
}

int rf_forward(void* h, float* kv, const uint32_t* tokens, uint32_t S, uint32_t pos,
               float* logits) {
    rf_model* m = h;
    if (!m || !kv || !tokens || !logits || S == 0 || pos + S > m->max_seq) return Q_ERR_INVALID_ARG;
    uint32_t D = m->dim, H = m->hidden, hd = D / m->n_heads, kvd = m->n_kv_heads * hd;
    size_t SD = (size_t)S * D;
    float *x = xalloc(SD * 4), *xn = xalloc(SD * 4), *q = xalloc(SD * 4), *qr = xalloc(SD * 4);
    float *k = xalloc((size_t)S * kvd * 4), *v = xalloc((size_t)S * kvd * 4);
    float *att = xalloc(SD * 4), *ao = xalloc(SD * 4), *mo = xalloc(SD * 4);
    float *g = xalloc((size_t)S * H * 4), *u = xalloc((size_t)S * H * 4);
    float *gs = xalloc((size_t)S * H * 4), *tmp = xalloc((size_t)hd * 4);
    float* lg = xalloc((size_t)m->vocab * 4);
    int rc = 0;
    for (uint32_t t = 0; t < S && !rc; t++) {
        if (tokens[t] >= m->vocab) rc = Q_ERR_INVALID_ARG;
        else memcpy(x + (size_t)t * D, m->token_embd + (size_t)tokens[t] * D, (size_t)D * 4);
    }
    size_t hs = (size_t)m->max_seq * 2 * hd, ls = hs * m->n_kv_heads;
    for (uint32_t l = 0; l < m->n_layers && !rc; l++) {
        for (uint32_t t = 0; t < S && !rc; t++)
            rc = q_rmsnorm_f32_avx2(x + (size_t)t * D, m->attn_norm[l], xn + (size_t)t * D, D, m->eps);
        for (uint32_t t = 0; t < S && !rc; t++) {
            rc = par_gemv(0, m->wq[l], D, D, xn + (size_t)t * D, q + (size_t)t * D);
            if (!rc) rc = par_gemv(0, m->wk[l], kvd, D, xn + (size_t)t * D, k + (size_t)t * kvd);
            if (!rc) rc = par_gemv(0, m->wv[l], kvd, D, xn + (size_t)t * D, v + (size_t)t * kvd);
        }
        for (uint32_t t = 0; t < S && !rc; t++) {
            const float* ct = m->cos_tab + (size_t)(pos + t) * hd;
            const float* st = m->sin_tab + (size_t)(pos + t) * hd;
            for (uint32_t hh = 0; hh < m->n_heads && !rc; hh++)
                rc = q_rope_f32_avx2(q + (size_t)t * D + hh * hd, ct, st, qr + (size_t)t * D + hh * hd, hd);
            for (uint32_t hh = 0; hh < m->n_kv_heads && !rc; hh++) {
                float* dst = kv + (size_t)l * ls + hh * hs + (size_t)(pos + t) * 2 * hd;
                rc = q_rope_f32_avx2(k + (size_t)t * kvd + hh * hd, ct, st, tmp, hd);
                memcpy(dst, tmp, (size_t)hd * 4);
                memcpy(dst + hd, v + (size_t)t * kvd + hh * hd, (size_t)hd * 4);
            }
        }
        if (rc) break;
        uint32_t items = S * m->n_heads;
        int nt = g_nt > (int)items ? (int)items : g_nt;
        attn_part ap[256];
        pthread_t th[256];
        uint32_t chunk = (items + (uint32_t)nt - 1) / (uint32_t)nt;
        int n = 0;
        for (int i = 0; i < nt; i++) {
            uint32_t lo = (uint32_t)i * chunk, hi = lo + chunk > items ? items : lo + chunk;
            if (lo >= hi) break;
            ap[n++] = (attn_part){m, kv, qr, att, S, pos, pos + S, hd, hs, (size_t)l * ls, lo, hi, 0};
        }
        for (int i = 1; i < n; i++) pthread_create(&th[i], NULL, attn_worker, &ap[i]);
        attn_worker(&ap[0]);
        for (int i = 1; i < n; i++) pthread_join(th[i], NULL);
        for (int i = 0; i < n; i++) if (ap[i].rc) rc = ap[i].rc;
        for (uint32_t t = 0; t < S && !rc; t++)
            rc = par_gemv(0, m->wo[l], D, D, att + (size_t)t * D, ao + (size_t)t * D);
        if (!rc) rc = vec_op(0, x, ao, x, SD);
        for (uint32_t t = 0; t < S && !rc; t++)
            rc = q_rmsnorm_f32_avx2(x + (size_t)t * D, m->ffn_norm[l], xn + (size_t)t * D, D, m->eps);
        for (uint32_t t = 0; t < S && !rc; t++) {
            rc = par_gemv(0, m->w_gate[l], H, D, xn + (size_t)t * D, g + (size_t)t * H);
            if (!rc) rc = par_gemv(0, m->w_up[l], H, D, xn + (size_t)t * D, u + (size_t)t * H);
        }
        if (!rc) rc = q_silu_f32_avx2(g, gs, S * H);
        if (!rc) rc = vec_op(1, gs, u, gs, (size_t)S * H);
        for (uint32_t t = 0; t < S && !rc; t++)
            rc = par_gemv(0, m->w_down[l], D, H, gs + (size_t)t * H, mo + (size_t)t * D);
        if (!rc) rc = vec_op(0, x, mo, x, SD);
    }
    if (!rc) rc = q_rmsnorm_f32_avx2(x + (size_t)(S - 1) * D, m->output_norm, xn, D, m->eps);
    if (!rc) rc = par_gemv(1, m->output, m->vocab, D, xn, lg);
    if (!rc) memcpy(logits, lg, (size_t)m->vocab * 4);
    free(x); free(xn); free(q); free(qr); free(k); free(v); free(att); free(ao); free(mo);
    free(g); free(u); free(gs); free(tmp); free(lg);
    return rc;
}
