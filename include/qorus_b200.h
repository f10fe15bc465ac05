/*
 * qorus_b200.h — additive entry points of libqorus_b200.so.
 *
 * The upstream API (qorus.h) is unchanged; nothing here is needed to use
 * it.  These calls exist for callers that want to keep data on the device
 * (device pointers in and out, an explicit CUDA stream), for the synthetic
 * model/KV generators the parity tests and benchmarks share, and for
 * tensor-parallel setup.  Streams are passed as `void*` (a cudaStream_t;
 * NULL = the legacy default stream) so the header needs no CUDA include.
 *
 * Each declaration names the upstream interface it stands beside.
 */
#ifndef QORUS_B200_H
#define QORUS_B200_H

#include "qorus.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- synthetic inputs (host, deterministic, multi-threaded) ------------
 * Counter-based: value i of stream s under seed k is a pure function of
 * (k, s, i), so any slice can be generated independently and the CPU
 * oracle and the device path see identical bytes.  Stand-in for the
 * upstream dummy-model writer tools/convert_llama.py:116-239, which wrote
 * FP32 noise where Q4_0 was expected; these write real Q4_0 blocks in the
 * [out][in] orientation (file order upstream src/models/model.c:355-619). */

/* Bytes of a .qorus v2 file for cfg (64-byte header + 64-byte padded tensors). */
size_t q_b200_model_file_size(const q_llama_config* cfg);

/* Write a random-init model: embeddings and output N(0,0.02), norm gains
 * 1+N(0,0.02), linear layers Q4_0 with nibbles uniform 0..15 and scales
 * uniform [0.001,0.01].  n_threads <= 0 means all online CPUs. */
q_error_code q_b200_write_model_file(const char* path, const q_llama_config* cfg,
                                     uint64_t seed, int n_threads);

/* out[j] = mean + stddev * N(0,1)[first_index + j] of stream `stream`. */
void q_b200_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream,
                        uint64_t first_index, float mean, float stddev, int n_threads);

/* out[j] = uniform integer in [0, modulus) drawn from (seed, stream, first_index+j). */
void q_b200_fill_tokens(uint32_t* out, size_t n, uint64_t seed, uint64_t stream,
                        uint64_t first_index, uint32_t modulus);

/* Q4_0 blocks with nibbles uniform 0..15 and scale uniform [smin, smax). */
void q_b200_fill_q4(q_block_q4_0* out, size_t n_blocks, uint64_t seed, uint64_t stream,
                    uint64_t first_block, float smin, float smax, int n_threads);

/* Fill positions [0, n_pos) of a HOST KV image in the upstream cache layout
 * [n_layers][n_kv_heads][max_seq_len][K(head_dim) | V(head_dim)] fp32
 * (upstream src/models/model.c:700-740) with N(0,1); other positions are
 * left untouched. */
q_error_code q_b200_fill_kv_prefill(float* kv_host, const q_llama_config* cfg,
                                    uint32_t n_pos, uint64_t seed, int n_threads);

/* ---- KV cache access (tier 2 lives in HBM) ----------------------------- */

/* Copy bytes between a host buffer and the device KV cache at a byte
 * offset into the upstream layout. */
q_error_code q_b200_kv_write(q_context* ctx, size_t offset, const void* host, size_t bytes);
q_error_code q_b200_kv_read(q_context* ctx, size_t offset, void* host, size_t bytes);

/* ---- device-resident decode -------------------------------------------- */

/* The CUDA stream every model kernel of this context runs on. */
void* q_b200_stream(q_context* ctx);

/* One greedy decode step like llama_forward(model, ctx, &token, 1, pos, …)
 * followed by q_sample_token(temperature 0), but the argmax runs on the
 * device and only the 4-byte token crosses PCIe. */
q_error_code q_b200_decode_greedy(q_llama_model* model, q_context* ctx, uint32_t token,
                                  uint32_t pos, uint32_t* next_token);

/* n_steps greedy decode steps replayed from the captured per-token CUDA
 * graph, the token fed back on the device; out_tokens[i] (host) receives
 * step i's argmax.  Asynchronous unless `sync` is non-zero; out_tokens is
 * written only when sync != 0. */
q_error_code q_b200_decode_loop(q_llama_model* model, q_context* ctx, uint32_t first_token,
                                uint32_t pos, uint32_t n_steps, uint32_t* out_tokens, int sync);

/* Profiling: one greedy decode step (as q_b200_decode_greedy) replayed from
 * a separately captured graph whose kernels stamp %globaltimer.  For each
 * kernel in launch order, out[3i..3i+2] = earliest CTA entry, earliest end
 * of its programmatic-dependency wait, latest exit (ns).  At most
 * max_kernels kernels are reported; *n_kernels receives the count.
 * Stands beside upstream's benchmark timing (tools/benchmark.c:22-50). */
q_error_code q_b200_profile_step(q_llama_model* model, q_context* ctx, uint32_t token,
                                 uint32_t pos, uint64_t* out, uint32_t max_kernels,
                                 uint32_t* n_kernels);

/* Device logits of the last forward / decode step ([vocab] fp32). */
const float* q_b200_device_logits(q_context* ctx);

/* ---- batched decode (several sequences per step) -----------------------
 * Upstream decodes one sequence per llama_forward call (qorus.h:212-219,
 * src/main.c:994-1131).  These calls decode up to 16 sequences together,
 * every weight streamed from HBM once per step for all of them.  Sequence b
 * has its own KV cache in the upstream layout [L][n_kv][max_seq][K|V]
 * (allocated by q_b200_batch_init, beside ctx's single-sequence cache),
 * after llama_build_graph.  On a tensor-parallel context every rank makes
 * the same calls (they are collective), each cache holds the rank's KV
 * heads, the partial residuals and argmax keys are all-reduced with NCCL,
 * and q_b200_decode_batch returns every rank the full [B][vocab] logits. */

/* Allocate the B caches (zeroed) and step state, capture the batched step. */
q_error_code q_b200_batch_init(q_context* ctx, q_llama_model* model, uint32_t batch);

/* The same with paged caches: one pool of n_pages pages, each holding
 * page_rows consecutive positions (a multiple of 32, or of 128 for head
 * width 32) of every layer and KV head.  A sequence takes pages as its rows
 * are written or decoded (each page zeroed when taken), so the pool can be
 * much smaller than batch * max_seq rows; q_b200_decode_batch(_loop) returns
 * Q_ERR_ARENA_OOM when it runs out.  q_b200_batch_kv_write/read keep the
 * upstream byte offsets (whole rows only in this mode; rows without a page
 * read as zeros). */
q_error_code q_b200_batch_init_paged(q_context* ctx, q_llama_model* model, uint32_t batch, uint32_t page_rows,
                                     uint32_t n_pages);

/* Give sequence seq's pages back to the pool (paged caches; a no-op for
 * contiguous ones): the slot starts empty for its next sequence. */
q_error_code q_b200_batch_release(q_context* ctx, uint32_t seq);

/* Copy bytes between a host buffer and sequence seq's cache (byte offset
 * into its upstream layout). */
q_error_code q_b200_batch_kv_write(q_context* ctx, uint32_t seq, size_t offset, const void* host,
                                   size_t bytes);
q_error_code q_b200_batch_kv_read(q_context* ctx, uint32_t seq, size_t offset, void* host, size_t bytes);

/* One greedy step of every sequence: token tokens[b] at position pos[b]
 * (attending to its cache positions 0..pos[b]).  logits (host, [B][vocab])
 * and next_tokens (host, [B], the argmax) may each be NULL. */
q_error_code q_b200_decode_batch(q_llama_model* model, q_context* ctx, const uint32_t* tokens,
                                 const uint32_t* pos, float* logits, uint32_t* next_tokens);

/* n_steps greedy steps from tokens / pos, each sequence's argmax fed back on
 * the device (graph replay); out_tokens[i * B + b] (host) receives step i's
 * token of sequence b.  Asynchronous unless sync != 0 (out_tokens written
 * only then). */
q_error_code q_b200_decode_batch_loop(q_llama_model* model, q_context* ctx, const uint32_t* tokens,
                                      const uint32_t* pos, uint32_t n_steps, uint32_t* out_tokens, int sync);

/* ---- tensor parallelism over the GPUs of one node ----------------------
 * No counterpart upstream (upstream is single-process).  One process per
 * GPU: rank 0 calls q_b200_tp_unique_id and shares the 128 bytes with the
 * others (any host channel); every rank then calls q_b200_tp_init with its
 * device current, after q_init_memory and before llama_build_graph.  Rank r
 * of W then uploads only its shard: query/KV heads [r*n/W, (r+1)*n/W) (its
 * KV cache holds those heads only, layout [L][n_kv/W][max_seq][K|V]), FFN
 * rows [r*H/W, ...) with the matching K-slices of wo and down, and vocab
 * rows [r*ceil(V/W), ...) of the LM head.  NCCL all-reduces the residual
 * after wo and down and the argmax key after the head; llama_forward
 * returns the full gathered logits on every rank.  Requires n_heads,
 * n_kv_heads and hidden_dim/32 divisible by W. */
q_error_code q_b200_tp_unique_id(void* id, size_t bytes);
q_error_code q_b200_tp_init(q_context* ctx, uint32_t rank, uint32_t world, const void* id, size_t bytes);

/* Optional, after q_b200_tp_init and before llama_build_graph: the decode
 * graph's all-reduces then run as one-shot exchanges over NVLink peer
 * memory instead of NCCL.  Each rank gets the CUDA IPC handle (64 bytes) of
 * its exchange buffer, the handles are shared in rank order over any host
 * channel, and each rank maps the others' buffers. */
q_error_code q_b200_tp_ipc_handle(q_context* ctx, void* handle, size_t bytes);
q_error_code q_b200_tp_ipc_open(q_context* ctx, const void* handles, size_t bytes);

/* Shard geometry of `rank` in `world` for cfg: out[0..12] = rank, world,
 * local q heads, local kv heads, q width, kv width, first q row, first kv
 * row, FFN width, first FFN row, vocab rows, first vocab row, rows per rank. */
q_error_code q_b200_tp_shape(const q_llama_config* cfg, uint32_t rank, uint32_t world, uint32_t* out,
                             uint32_t n);

/* ---- kernel entry points on device buffers ------------------------------
 * The Q4_0 GEMV of upstream src/ops/avx2/matmul.c:98-271 on device memory.
 * Weights are first repacked from the upstream 20-byte AoS blocks into the
 * device stream layout (tiles of rows; 16-byte nibble planes then fp32
 * scales per tile). */
size_t q_b200_q4_packed_bytes(uint32_t M, uint32_t K);
q_error_code q_b200_q4_pack(const q_block_q4_0* d_src, uint32_t M, uint32_t K,
                            void* d_dst, void* stream);
q_error_code q_b200_gemv_q4(const void* d_packed, uint32_t M, uint32_t K,
                            const float* d_x, float* d_y, void* stream);

/* Same GEMV as q_b200_gemv_q4, for callers that may not allocate device
 * memory: no cudaMalloc/cudaFree ever; split-slab scratch is a fixed 2 MiB
 * device array of the library.  The first call on a device (device current)
 * resolves that array and must precede any stream capture meant to hold the
 * launch; shapes needing more scratch return Q_ERR_INVALID_SIZE; calls that
 * can overlap on one device race on the shared scratch and must be
 * serialised by the caller.  No counterpart in the reference. */
q_error_code q_b200_gemv_q4_noalloc(const void* d_packed, uint32_t M, uint32_t K,
                                    const float* d_x, float* d_y, void* stream);

/* The same Q4_0 product over n_rows input rows at once: d_y[r][m] =
 * sum_k W[m][k] d_x[r][k] for r < n_rows (d_x [n_rows][K], d_y [n_rows][M],
 * fp32, 16-byte aligned).  This is the prompt-path contraction: upstream
 * runs q_gemv_q4_f32_avx2 (src/ops/avx2/matmul.c:98-271) once per prompt
 * row (src/models/model.c:1120-1165); here the rows go through one
 * tensor-core GEMM (tcgen05) with fp16 hi/lo operand halves (an fp32-grade
 * result).  Allocates a workspace on first use (grown, then kept). */
q_error_code q_b200_gemm_q4(const void* d_packed, uint32_t M, uint32_t K, const float* d_x,
                            uint32_t n_rows, float* d_y, void* stream);

/* FP32 GEMV y[M] = W[M,K] x[K] (the LM head of upstream
 * src/models/model.c:1821-1844, dot order of src/ops/avx2/matmul_fp32.c). */
q_error_code q_b200_gemv_f32(const float* d_w, uint32_t M, uint32_t K,
                             const float* d_x, float* d_y, void* stream);

/* ---- device errors and bounded waits -------------------------------------
 * No counterpart upstream (upstream's kernels run on the calling thread and
 * cannot hang).  Every device-side wait of this library (a copy that should
 * land in shared memory, a grid barrier, a peer rank's flag) is bounded in
 * wall time; when one runs out the kernel records a code in a per-device
 * status word and returns, and the upstream-API calls that synchronise
 * (llama_forward, q_generate, q_b200_decode_loop with sync) report it as
 * Q_ERR_INVALID_ARG with the message in q_b200_last_error().  The
 * device-pointer entry points (q_b200_gemv_q4, q_b200_gemv_q4_noalloc, ...)
 * are asynchronous and cannot: after synchronising their stream, read the
 * word with q_b200_device_status. */

/* Wall-time limit of every bounded device wait on the current device, in
 * ns (default 2 s).  Applies to kernels launched after the call. */
q_error_code q_b200_set_wait_limit_ns(uint64_t ns);

/* Status word of the current device: 0 if no wait ran out since the last
 * read, else the code of the first one (1-3 copy waits, 5 grid barrier,
 * 6 peer flag).  Reading clears it; when it was set, this first waits for
 * all work on the device and re-zeroes the library's ticket and barrier
 * counters, which a wait that gave up can leave non-zero. */
uint32_t q_b200_device_status(void);

/* Self-test of the failure path: launches the fused tensor-parallel
 * receive GEMV on the current device alone, with an exchange buffer no
 * sender ever writes, under a wait limit of limit_ns (restored afterwards).
 * Every CTA's flag wait runs out; *status_out receives the status word
 * observed (6 = peer flag timeout), which is then cleared.  Returns Q_OK
 * when the launch completed and the context is still usable. */
q_error_code q_b200_selftest_exchange_timeout(uint64_t limit_ns, uint32_t* status_out);

/* Number of kernels this library launched since load (all entry points). */
uint64_t q_b200_kernel_launches(void);

/* Number of device allocations (cudaMalloc) this library made since load. */
uint64_t q_b200_device_allocations(void);

/* Last CUDA error string seen by the library ("" if none). */
const char* q_b200_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* QORUS_B200_H */
