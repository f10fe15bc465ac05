/*
 * qorus.h — the Qorus-IA public C API, served by libqorus_b200.so.
 *
 * Names, argument order, argument meaning and return codes are those of the
 * upstream header (jcopari/Project-IA include/qorus.h); the cited line is the
 * upstream declaration each entry point replaces.  The work behind them runs
 * on an NVIDIA B200 (sm_100a): the three memory tiers live in HBM, the model
 * forward is a chain of hand-written CUDA kernels, and every call is
 * synchronous for the caller (host buffers in, host buffers out) exactly as
 * upstream.  There is no CPU fallback: with no usable GPU the entry points
 * return Q_ERR_INVALID_ARG (or Q_ERR_ALLOC_FAILED for allocations).
 */
#ifndef QORUS_H
#define QORUS_H

#include "qorus_types.h"

#ifdef __cplusplus
#define Q_RESTRICT __restrict__
extern "C" {
#else
#define Q_RESTRICT restrict
#endif

/* ---- memory tiers (upstream src/core/memory.c) ------------------------ */

/* upstream include/qorus.h:16 — mmap the model file (tier 1, host). */
q_error_code q_init_memory(q_context* Q_RESTRICT ctx, const char* model_path);

/* upstream include/qorus.h:21 — same, with an mmap strategy. */
q_error_code q_init_memory_ex(q_context* Q_RESTRICT ctx, const char* model_path,
                              q_mmap_strategy strategy);

/* upstream include/qorus.h:25 — tier 2: allocates kv_size bytes of HBM,
 * zeroed; ctx->kv_buffer becomes a device pointer. */
q_error_code q_alloc_kv_cache(q_context* Q_RESTRICT ctx, size_t kv_size);

/* upstream include/qorus.h:29 — tier 3: a host arena (views, model structs)
 * and a device arena of the same size for activations. */
q_error_code q_alloc_arena(q_context* Q_RESTRICT ctx, size_t arena_size);

/* upstream include/qorus.h:33 — 64-byte aligned bump allocation (host). */
void* q_arena_alloc(q_context* Q_RESTRICT ctx, size_t size);

/* upstream include/qorus.h:36 — rewind both arenas to the watermark. */
void q_arena_reset(q_context* Q_RESTRICT ctx);

/* upstream include/qorus.h:39 — free device state, arena, KV cache, mmap. */
void q_free_memory(q_context* Q_RESTRICT ctx);

/* upstream include/qorus.h:47 */
const char* q_strerror(q_error_code err);

/* ---- kernel-level entry points (host buffers; run on the GPU) ---------- */

/* upstream include/qorus.h:58 — one Q4_0 block to 32 floats. */
void q_dequantize_q4_0_block_avx2_public(const q_block_q4_0* Q_RESTRICT block,
                                         float* Q_RESTRICT output);

/* upstream include/qorus.h:70 — y[M] = deq(W[M, N]) x[N]; W is a Q4_0 view
 * with ne[0]=M rows, ne[1]=N columns (N % 32 == 0), nb[0] = N/32*20. */
q_error_code q_gemv_q4_f32_avx2(const q_tensor* Q_RESTRICT weights,
                                const float* Q_RESTRICT input,
                                float* Q_RESTRICT output);

/* upstream include/qorus.h:84 — C[M,N] = A[M,K] B[K,N] (FP32). */
q_error_code q_matmul_f32_avx2(const q_tensor* Q_RESTRICT A, const q_tensor* Q_RESTRICT B,
                               q_tensor* C, q_context* Q_RESTRICT ctx);

/* upstream include/qorus.h:97 */
q_error_code q_causal_mask_f32_avx2(q_tensor* scores, float mask_value);

/* upstream include/qorus.h:109 */
q_error_code q_add_f32_avx2(const q_tensor* a, const q_tensor* b, q_tensor* output);

/* upstream include/qorus.h:122 */
q_error_code q_mul_f32_avx2(const q_tensor* a, const q_tensor* b, q_tensor* output);

/* upstream include/qorus.h:138 */
q_error_code q_rmsnorm_f32_avx2(const float* Q_RESTRICT x, const float* Q_RESTRICT weight,
                                float* Q_RESTRICT output, uint32_t N, float eps);

/* upstream include/qorus.h:153 — interleaved-pair rotation, duplicated
 * cos/sin tables ([c0,c0,c1,c1,...]). */
q_error_code q_rope_f32_avx2(const float* Q_RESTRICT x, const float* Q_RESTRICT cos,
                             const float* Q_RESTRICT sin, float* Q_RESTRICT output,
                             uint32_t N);

/* upstream include/qorus.h:167 */
q_error_code q_silu_f32_avx2(const float* Q_RESTRICT x, float* Q_RESTRICT output, uint32_t N);

/* upstream include/qorus.h:179 */
q_error_code q_softmax_f32_avx2(const float* Q_RESTRICT x, float* Q_RESTRICT output, uint32_t N);

/* ---- Llama-3 model (upstream src/models/model.c) ----------------------- */

/* upstream include/qorus.h:193 — validate the header, build host views,
 * then upload the weights once to HBM (Q4_0 repacked into the device
 * stream layout) and capture the per-token CUDA graph. */
q_error_code llama_build_graph(q_context* Q_RESTRICT ctx, q_llama_model* Q_RESTRICT model);

/* upstream include/qorus.h:200 — nulls the model pointers; device weights
 * are released by q_free_memory. */
void llama_free_graph(q_llama_model* Q_RESTRICT model);

/* upstream include/qorus.h:212 — run tokens[0..seq_len) at positions
 * pos..pos+seq_len-1 through the model, writing K/V into the cache, and
 * copy the last row's logits[vocab] to the host buffer. */
q_error_code llama_forward(q_llama_model* Q_RESTRICT model, q_context* Q_RESTRICT ctx,
                           const uint32_t* Q_RESTRICT tokens, uint32_t seq_len,
                           uint32_t pos, float* Q_RESTRICT logits);

/* ---- generation (upstream src/main.c) ---------------------------------- */

/* upstream include/qorus.h:292 — greedy when temperature < 1e-6 (first
 * index of the maximum); otherwise temperature, top-k, top-p and one draw of
 * the per-thread xorshift64* stream, computed on the device. */
q_error_code q_sample_token(const float* Q_RESTRICT logits, uint32_t vocab_size,
                            float temperature, uint32_t top_k, float top_p,
                            uint32_t* Q_RESTRICT token_id_out, q_context* Q_RESTRICT ctx);

/* upstream include/qorus.h:318 — prefill, then decode with greedy argmax or
 * the sampler on the device, so no logits cross PCIe per token. */
q_error_code q_generate(q_generation_state* Q_RESTRICT state);

/* ---- tokenizer (upstream src/tokenizer/bpe.c, host code) --------------- */

/* upstream include/qorus.h:230 — read a 'QTKR' v1 tokenizer file. */
q_error_code q_tokenizer_load(q_tokenizer* Q_RESTRICT tok, const char* tokenizer_path);

/* upstream include/qorus.h:242 — byte ids, greedy BPE merges in rule order,
 * optional BOS/EOS; Q_ERR_ARENA_OOM when the result exceeds max_tokens. */
q_error_code q_tokenizer_encode(q_tokenizer* Q_RESTRICT tok, const char* Q_RESTRICT text,
                                uint32_t* Q_RESTRICT tokens_out, uint32_t* Q_RESTRICT num_tokens_out,
                                uint32_t max_tokens, bool add_bos, bool add_eos);

/* upstream include/qorus.h:260 — concatenated token strings, special and
 * out-of-range ids skipped; Q_ERR_ARENA_OOM (truncated) when it does not fit. */
q_error_code q_tokenizer_decode(q_tokenizer* Q_RESTRICT tok, const uint32_t* Q_RESTRICT tokens,
                                uint32_t num_tokens, char* Q_RESTRICT text_out, size_t text_buf_size);

/* upstream include/qorus.h:273 — release everything and zero the struct. */
void q_tokenizer_free(q_tokenizer* Q_RESTRICT tok);

#ifdef __cplusplus
}
#endif

#endif /* QORUS_H */
