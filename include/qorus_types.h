/*
 * qorus_types.h — data types of the Qorus-IA C API, B200 build.
 *
 * Every type here is ABI-identical to the upstream declaration it replaces
 * (include/qorus_types.h of jcopari/Project-IA), so a caller compiled
 * against the upstream header links against libqorus_b200.so unchanged:
 *   q_error_code        upstream include/qorus_types.h:30-48
 *   q_mmap_strategy     upstream include/qorus_types.h:54-57
 *   q_dtype             upstream include/qorus_types.h:134-138
 *   q_tokenizer         upstream include/qorus_types.h:145-175
 *   q_block_q4_0        upstream include/qorus_types.h:183-186
 *   q_model_header      upstream include/qorus_types.h:189-203
 *   q_tensor            upstream include/qorus_types.h:206-213
 *   q_context           upstream include/qorus_types.h:216-231
 *   q_llama_config/layer/model, q_generation_state
 *                       upstream include/qorus_types.h:238-306
 *
 * Differences in meaning (not in layout) for the B200 build:
 *   q_context.kv_buffer   is a DEVICE pointer (cudaMalloc'd HBM).  Host code
 *                         must not dereference it; use q_b200_kv_read/write.
 *   q_context.scratch_*   stay a HOST arena (tensor views, model structs, as
 *                         upstream).  A device arena of the same size is
 *                         allocated beside it and reset with it.
 */
#ifndef QORUS_TYPES_H
#define QORUS_TYPES_H

#include <stdint.h>
#include <stddef.h>
#include <stdbool.h>
#include <stdio.h>

#define Q_ALIGN 64
#define Q_MAGIC 0x514F5231u            /* 'QOR1' little-endian */
#define Q_HEADER_SIZE 64
#define Q_FIRST_TENSOR_OFFSET Q_HEADER_SIZE
#define Q_ALIGN_SIZE(size) (((size) + Q_ALIGN - 1) & ~((size_t)Q_ALIGN - 1))

/* Tolerances the upstream tests use. */
#define Q_EPSILON_ABS_F32    1e-5f
#define Q_EPSILON_REL_F32    1e-4f
#define Q_EPSILON_ABS_APPROX 2.5e-1f
#define Q_EPSILON_REL_APPROX 5e-1f
#define Q_EPSILON_ABS_Q4_VAL 1e-2f
#define Q_EPSILON_REL_Q4_VAL 5e-2f

typedef enum {
    Q_OK = 0,
    Q_ERR_NULL_PTR = -1,
    Q_ERR_FILE_OPEN = -2,
    Q_ERR_FILE_STAT = -3,
    Q_ERR_FILE_TOO_SMALL = -4,
    Q_ERR_MMAP_FAILED = -5,
    Q_ERR_INVALID_MAGIC = -6,
    Q_ERR_ALLOC_FAILED = -7,   /* also: cudaMalloc failed */
    Q_ERR_ARENA_OOM = -8,      /* also: device arena exhausted */
    Q_ERR_INVALID_CONFIG = -9,
    Q_ERR_INVALID_ARG = -10,   /* also: a CUDA launch/runtime error */
    Q_ERR_ALIASING = -11,
    Q_ERR_OVERFLOW = -12,
    Q_ERR_MISALIGNED = -13,
    Q_ERR_INVALID_DTYPE = -14,
    Q_ERR_INVALID_SIZE = -15
} q_error_code;

typedef enum {
    Q_MMAP_LAZY = 0,
    Q_MMAP_EAGER = 1
} q_mmap_strategy;

typedef enum {
    Q_F32 = 0,
    Q_Q8_0 = 1,
    Q_Q4_0 = 2
} q_dtype;

typedef struct {
    uint32_t token_id1;
    uint32_t token_id2;
    uint32_t merged_id;
} q_bpe_merge;

struct bpe_hash_table;

typedef struct {
    char** vocab;
    uint32_t vocab_size;
    q_bpe_merge* merges;
    uint32_t num_merges;
    struct bpe_hash_table* merge_hash_table;
    uint32_t bos_token_id;
    uint32_t eos_token_id;
    uint32_t pad_token_id;
    bool initialized;
} q_tokenizer;

/* One Q4_0 block: 32 weights.  Byte b of qs holds weight 2b in its low
 * nibble and weight 2b+1 in its high nibble; weight = (nibble - 8) * scale. */
typedef struct {
    uint8_t qs[16];
    float scale;
} __attribute__((packed)) q_block_q4_0;

/* 64-byte file header of a .qorus model file. */
typedef struct {
    uint32_t magic;
    uint32_t version;
    uint32_t vocab_size;
    uint32_t dim;
    uint32_t hidden_dim;
    uint32_t n_layers;
    uint32_t n_heads;
    uint32_t n_kv_heads;
    uint32_t max_seq_len;
    float rope_freq_base;
    float rms_norm_eps;        /* read when version >= 2 */
    uint32_t reserved[5];
} __attribute__((packed, aligned(64))) q_model_header;

typedef struct {
    void* data;
    float* scales;
    uint32_t ne[4];
    size_t nb[4];
    q_dtype type;
    char name[32];
} __attribute__((aligned(Q_ALIGN))) q_tensor;

typedef struct {
    /* tier 1: the mmapped model file (host) */
    void* weights_mmap;
    size_t weights_size;
    q_model_header* header;
    /* tier 2: KV cache — device memory in this build */
    void* kv_buffer;
    size_t kv_size;
    /* tier 3: bump arena (host views); a device twin is kept internally */
    void* scratch_buffer;
    size_t scratch_size;
    size_t scratch_head;
    size_t scratch_base_offset;
} q_context;

typedef struct {
    uint32_t vocab_size;
    uint32_t dim;
    uint32_t hidden_dim;
    uint32_t n_layers;
    uint32_t n_heads;
    uint32_t n_kv_heads;
    uint32_t max_seq_len;
    float rope_freq_base;
    float rms_norm_eps;
} q_llama_config;

typedef struct {
    uint32_t layer_idx;
    q_tensor* attn_norm;
    q_tensor* wq;
    q_tensor* wk;
    q_tensor* wv;
    q_tensor* wo;
    q_tensor* ffn_norm;
    q_tensor* w_gate;
    q_tensor* w_up;
    q_tensor* w_down;
} q_llama_layer;

typedef struct {
    q_llama_config config;
    q_tensor* token_embd;
    q_tensor* output_norm;
    q_tensor* output;
    q_llama_layer* layers;
    float* rope_freqs;
    bool rope_cache_enabled;
    float* rope_cos_cache;
    float* rope_sin_cache;
    q_context* ctx;
} q_llama_model;

typedef struct {
    q_context* ctx;
    q_llama_model* model;
    q_tokenizer* tokenizer;
    uint32_t* prompt_tokens;
    uint32_t num_prompt_tokens;
    uint32_t* generated_tokens;
    uint32_t num_generated_tokens;
    uint32_t max_tokens;
    float temperature;
    uint32_t top_k;
    float top_p;
    uint32_t current_pos;
} q_generation_state;

#endif /* QORUS_TYPES_H */
