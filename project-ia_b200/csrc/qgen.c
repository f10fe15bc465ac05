/*
 * qgen.c — deterministic synthetic model / KV / token generators (host).
 *
 * Every value is a pure function of (seed, stream, index) through a
 * SplitMix64 mix, so threads fill disjoint slices in any order and the
 * CPU oracle and the device path read identical bytes.  Normals come from
 * the Box–Muller transform on pairs (2k, 2k+1) of 24-bit uniforms.
 *
 * The .qorus layout written here is the one upstream llama_build_graph
 * reads (src/models/model.c:355-619): 64-byte header, then token_embd
 * [vocab][dim] f32, output_norm [dim], output [vocab][dim] f32, then per
 * layer attn_norm, wq, wk, wv, wo, ffn_norm, w_gate, w_up, w_down, every
 * tensor padded to 64 bytes.  Linear weights are stored [out][in]: row r
 * holds in/32 Q4_0 blocks (byte sizes equal the upstream ones, which only
 * depend on rows*cols).  Header version 2 carries rms_norm_eps
 * (include/qorus_types.h:189-203 upstream).
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "qorus_b200.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t stream_base(uint64_t seed, uint64_t stream) {
    return mix64(seed ^ mix64(stream * 0xD1B54A32D192ED03ull + 0x1234567ull));
}

static inline uint64_t draw(uint64_t base, uint64_t i) {
    return mix64(base + i * 0x9E3779B97F4A7C15ull);
}

static inline float u24(uint64_t h) { return (float)(h >> 40) * (1.0f / 16777216.0f); }

static inline float normal_at(uint64_t base, uint64_t i) {
    uint64_t k = i >> 1;
    float u1 = ((float)(draw(base, 2 * k) >> 40) + 1.0f) * (1.0f / 16777216.0f);
    float u2 = u24(draw(base, 2 * k + 1));
    float r = sqrtf(-2.0f * logf(u1));
    float th = 6.28318530717958647692f * u2;
    return (i & 1) ? r * sinf(th) : r * cosf(th);
}

static int online_cpus(int n) {
    if (n > 0) return n;
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    if (c < 1) c = 1;
    if (c > 256) c = 256;
    return (int)c;
}

/* ---- threaded range helper -------------------------------------------- */

typedef void (*range_fn)(void* arg, size_t lo, size_t hi);
typedef struct { range_fn fn; void* arg; size_t lo, hi; } range_job;

static void* range_thread(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->arg, j->lo, j->hi);
    return NULL;
}

static void parallel_range(range_fn fn, void* arg, size_t n, int n_threads) {
    int t = online_cpus(n_threads);
    if (n < (size_t)1 << 16 || t == 1) { fn(arg, 0, n); return; }
    if ((size_t)t > n) t = (int)n;
    pthread_t th[256];
    range_job jobs[256];
    size_t chunk = (n + (size_t)t - 1) / (size_t)t;
    int started = 0;
    for (int i = 0; i < t; i++) {
        size_t lo = (size_t)i * chunk, hi = lo + chunk > n ? n : lo + chunk;
        if (lo >= hi) break;
        jobs[i] = (range_job){fn, arg, lo, hi};
        if (pthread_create(&th[i], NULL, range_thread, &jobs[i]) != 0) {
            fn(arg, lo, hi);
            jobs[i].fn = NULL;
        }
        started = i + 1;
    }
    for (int i = 0; i < started; i++)
        if (jobs[i].fn) pthread_join(th[i], NULL);
}

/* ---- normals ----------------------------------------------------------- */

typedef struct { float* out; uint64_t base, first; float mean, sd; } normal_job;

static void normal_range(void* a, size_t lo, size_t hi) {
    normal_job* j = (normal_job*)a;
    for (size_t i = lo; i < hi; i++)
        j->out[i] = j->mean + j->sd * normal_at(j->base, j->first + i);
}

void q_b200_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream,
                        uint64_t first_index, float mean, float stddev, int n_threads) {
    if (!out || n == 0) return;
    normal_job j = {out, stream_base(seed, stream), first_index, mean, stddev};
    parallel_range(normal_range, &j, n, n_threads);
}

void q_b200_fill_tokens(uint32_t* out, size_t n, uint64_t seed, uint64_t stream,
                        uint64_t first_index, uint32_t modulus) {
    if (!out || modulus == 0) return;
    uint64_t base = stream_base(seed, stream);
    for (size_t i = 0; i < n; i++)
        out[i] = (uint32_t)(draw(base, first_index + i) % modulus);
}

/* ---- Q4_0 blocks --------------------------------------------------------- */

typedef struct { q_block_q4_0* out; uint64_t bq, bs, first; float smin, span; } q4_job;

static void q4_range(void* a, size_t lo, size_t hi) {
    q4_job* j = (q4_job*)a;
    for (size_t i = lo; i < hi; i++) {
        uint64_t g = j->first + i;
        uint64_t h0 = draw(j->bq, 2 * g), h1 = draw(j->bq, 2 * g + 1);
        q_block_q4_0 blk;
        memcpy(blk.qs, &h0, 8);
        memcpy(blk.qs + 8, &h1, 8);
        blk.scale = j->smin + j->span * u24(draw(j->bs, g));
        memcpy(&j->out[i], &blk, sizeof blk);
    }
}

void q_b200_fill_q4(q_block_q4_0* out, size_t n_blocks, uint64_t seed, uint64_t stream,
                    uint64_t first_block, float smin, float smax, int n_threads) {
    if (!out || n_blocks == 0) return;
    q4_job j = {out, stream_base(seed, stream), stream_base(seed, stream ^ (1ull << 40)),
                first_block, smin, smax - smin};
    parallel_range(q4_range, &j, n_blocks, n_threads);
}

/* ---- model file ------------------------------------------------------------ */

static size_t f32_bytes(size_t n) { return Q_ALIGN_SIZE(n * sizeof(float)); }
static size_t q4_bytes(size_t rows, size_t cols) { return Q_ALIGN_SIZE(rows * (cols / 32) * 20); }

static int cfg_ok(const q_llama_config* c) {
    return c && c->vocab_size && c->dim && c->hidden_dim && c->n_layers && c->n_heads &&
           c->n_kv_heads && c->dim % 32 == 0 && c->hidden_dim % 32 == 0 &&
           c->dim % c->n_heads == 0 && c->n_heads % c->n_kv_heads == 0;
}

size_t q_b200_model_file_size(const q_llama_config* c) {
    if (!cfg_ok(c)) return 0;
    size_t D = c->dim, H = c->hidden_dim, V = c->vocab_size;
    size_t kv = (size_t)c->n_kv_heads * (D / c->n_heads);
    size_t layer = 2 * f32_bytes(D) + 2 * q4_bytes(D, D) + 2 * q4_bytes(kv, D) +
                   2 * q4_bytes(H, D) + q4_bytes(D, H);
    return Q_HEADER_SIZE + 2 * f32_bytes(V * D) + f32_bytes(D) + layer * c->n_layers;
}

q_error_code q_b200_write_model_file(const char* path, const q_llama_config* c,
                                     uint64_t seed, int n_threads) {
    if (!path || !c) return Q_ERR_NULL_PTR;
    if (!cfg_ok(c)) return Q_ERR_INVALID_CONFIG;
    size_t total = q_b200_model_file_size(c);
    int fd = open(path, O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return Q_ERR_FILE_OPEN;
    if (ftruncate(fd, (off_t)total) != 0) { close(fd); return Q_ERR_ALLOC_FAILED; }
    uint8_t* m = (uint8_t*)mmap(NULL, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return Q_ERR_MMAP_FAILED;

    q_model_header h;
    memset(&h, 0, sizeof h);
    h.magic = Q_MAGIC;
    h.version = 2;
    h.vocab_size = c->vocab_size;
    h.dim = c->dim;
    h.hidden_dim = c->hidden_dim;
    h.n_layers = c->n_layers;
    h.n_heads = c->n_heads;
    h.n_kv_heads = c->n_kv_heads;
    h.max_seq_len = c->max_seq_len;
    h.rope_freq_base = c->rope_freq_base;
    h.rms_norm_eps = c->rms_norm_eps;
    memcpy(m, &h, sizeof h);

    size_t D = c->dim, H = c->hidden_dim, V = c->vocab_size;
    size_t kv = (size_t)c->n_kv_heads * (D / c->n_heads);
    size_t off = Q_HEADER_SIZE;
    uint64_t stream = 0;
#define EMIT_NORMAL(n, mean, sd)                                                   \
    do {                                                                           \
        q_b200_fill_normal((float*)(m + off), (n), seed, stream, 0, (mean), (sd),  \
                           n_threads);                                             \
        off += f32_bytes(n);                                                       \
        stream++;                                                                  \
    } while (0)
#define EMIT_Q4(rows, cols)                                                            \
    do {                                                                               \
        q_b200_fill_q4((q_block_q4_0*)(m + off), (rows) * ((cols) / 32), seed, stream, \
                       0, 0.001f, 0.01f, n_threads);                                   \
        off += q4_bytes(rows, cols);                                                   \
        stream++;                                                                      \
    } while (0)
    EMIT_NORMAL(V * D, 0.0f, 0.02f); /* token_embd */
    EMIT_NORMAL(D, 1.0f, 0.02f);     /* output_norm */
    EMIT_NORMAL(V * D, 0.0f, 0.02f); /* output */
    for (uint32_t l = 0; l < c->n_layers; l++) {
        EMIT_NORMAL(D, 1.0f, 0.02f); /* attn_norm */
        EMIT_Q4(D, D);               /* wq */
        EMIT_Q4(kv, D);              /* wk */
        EMIT_Q4(kv, D);              /* wv */
        EMIT_Q4(D, D);               /* wo */
        EMIT_NORMAL(D, 1.0f, 0.02f); /* ffn_norm */
        EMIT_Q4(H, D);               /* w_gate */
        EMIT_Q4(H, D);               /* w_up */
        EMIT_Q4(D, H);               /* w_down */
    }
#undef EMIT_NORMAL
#undef EMIT_Q4
    int bad = off != total;
    munmap(m, total);
    return bad ? Q_ERR_OVERFLOW : Q_OK;
}

/* ---- KV image ---------------------------------------------------------------- */

#define Q_KV_STREAM 0x4B56ull /* 'KV' */

q_error_code q_b200_fill_kv_prefill(float* kv, const q_llama_config* c, uint32_t n_pos,
                                    uint64_t seed, int n_threads) {
    if (!kv || !c) return Q_ERR_NULL_PTR;
    if (!cfg_ok(c) || n_pos > c->max_seq_len) return Q_ERR_INVALID_SIZE;
    size_t hd = c->dim / c->n_heads, row = 2 * hd;
    for (size_t l = 0; l < c->n_layers; l++)
        for (size_t h = 0; h < c->n_kv_heads; h++) {
            size_t slab = l * c->n_kv_heads + h;
            float* dst = kv + slab * (size_t)c->max_seq_len * row;
            q_b200_fill_normal(dst, (size_t)n_pos * row, seed, Q_KV_STREAM,
                               (uint64_t)slab * n_pos * row, 0.0f, 1.0f, n_threads);
        }
    return Q_OK;
}
