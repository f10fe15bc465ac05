/*
 * oracle.h — CPU restatement of the Qorus-IA Llama-3 forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the parity tests, the
 * smoke test and bench.py's cpu_baseline leg compare the CUDA path against;
 * nothing in the product links or calls it.
 *
 * Each function restates one upstream function (jcopari/Project-IA, path
 * relative to that repository), keeping its arithmetic: the same 8-lane x
 * 4-accumulator summation orders, the same polynomial exp on the same
 * element indices with libm expf on the tails, the same unfused mul/add
 * where upstream does not use FMA.  The forward composes these kernels into
 * the intended Llama-3 graph: [out][in] weights, per-row RMSNorm, attention
 * over KV-cache positions 0..pos+t with GQA, as the upstream graph intends
 * but only implements for square shapes at seq_len 1.
 */
#ifndef QORUS_ORACLE_H
#define QORUS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/ops/avx2/avx_math.h:10-61 */
float orc_exp_approx(float x);

/* src/ops/avx2/dequantize.c:18-73 — 20-byte block to 32 floats. */
void orc_dequantize_block(const uint8_t* block20, float* out32);

/* src/ops/avx2/matmul.c:43-271 — y[M] = deq(W[M][K]) x[K], W as upstream
 * 20-byte AoS blocks, K % 32 == 0. */
int orc_gemv_q4(const uint8_t* w, uint32_t M, uint32_t K, const float* x, float* y);

/* src/ops/avx2/matmul_fp32.c:302-471 — one output of the FP32 matmul:
 * dot(a, b) over K with 4 x 8-lane FMA accumulators on K & ~31 and an
 * unfused scalar tail. */
float orc_dot_f32(const float* a, const float* b, uint32_t K);

/* y[M] = W[M][K] x[K] through orc_dot_f32 (the LM head, model.c:1821-1844). */
int orc_gemv_f32(const float* w, uint32_t M, uint32_t K, const float* x, float* y);

/* src/ops/avx2/rmsnorm.c:15-92 (N % 8 == 0).  The hardware rsqrt estimate
 * of upstream is replaced by 1/sqrtf before the same Newton step. */
int orc_rmsnorm(const float* x, const float* w, float* out, uint32_t N, float eps);

/* src/ops/avx2/rope.c:23-110 (N % 8 == 0, duplicated tables). */
int orc_rope(const float* x, const float* c, const float* s, float* out, uint32_t N);

/* src/ops/avx2/softmax.c:17-132 */
int orc_softmax(const float* x, float* out, uint32_t N);

/* src/ops/avx2/silu.c:18-94 */
int orc_silu(const float* x, float* out, uint32_t N);

/* src/models/model.c:625-665 — duplicated cos/sin tables [max_seq][hd]. */
void orc_rope_tables(float theta, uint32_t head_dim, uint32_t max_seq, float* cos_tab,
                     float* sin_tab);

/* Parsed .qorus file (pointers into caller-owned file bytes). */
typedef struct {
    uint32_t vocab, dim, hidden, n_layers, n_heads, n_kv_heads, max_seq;
    float theta, eps;
    const float* token_embd;
    const float* output_norm;
    const float* output;
    const float* attn_norm[512];
    const uint8_t* wq[512];
    const uint8_t* wk[512];
    const uint8_t* wv[512];
    const uint8_t* wo[512];
    const float* ffn_norm[512];
    const uint8_t* w_gate[512];
    const uint8_t* w_up[512];
    const uint8_t* w_down[512];
    float* cos_tab;  /* owned, [max_seq][hd] */
    float* sin_tab;
} orc_model;

/* Parse header + tensor offsets (src/models/model.c:294-673).  Returns 0 or
 * a negative q_error_code value. */
int orc_model_open(orc_model* m, const void* file, size_t size);
void orc_model_close(orc_model* m);

/* Intended Llama-3 forward of tokens[0..S) at positions pos..pos+S-1.
 * kv is the host cache image [L][n_kv][max_seq][K|V] (updated).  logits
 * receives the last row's vocab logits. */
int orc_forward(const orc_model* m, float* kv, const uint32_t* tokens, uint32_t S,
                uint32_t pos, float* logits);

/* First index of the maximum (src/main.c:870-881). */
uint32_t orc_argmax(const float* x, uint32_t n);

/* Worker threads for the row-parallel loops (results do not depend on it). */
void orc_set_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
