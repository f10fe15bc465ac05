// api_model.cu — llama_build_graph / llama_forward / q_generate on the B200,
// and the device-resident decode entry points of qorus_b200.h.
#include <cmath>
#include <cstdlib>

#include "runtime.cuh"

using namespace qb200;

static size_t al64(size_t n) { return (n + 63) & ~(size_t)63; }

// Host tensor view in the host arena, bounds-checked against the mmap
// (upstream create_tensor_view, model.c:170-292).  Views use the [out][in]
// orientation the device kernels read (ne[0] = rows, ne[1] = columns).
static q_tensor* make_view(q_context* ctx, size_t off, uint32_t ne0, uint32_t ne1, q_dtype t,
                           const char* name) {
    size_t bytes = t == Q_F32 ? (size_t)ne0 * ne1 * 4 : (size_t)ne0 * (ne1 / 32) * 20;
    if (bytes == 0 || off + bytes > ctx->weights_size) return nullptr;
    q_tensor* v = (q_tensor*)q_arena_alloc(ctx, sizeof(q_tensor));
    if (!v) return nullptr;
    memset(v, 0, sizeof *v);
    v->data = (uint8_t*)ctx->weights_mmap + off;
    v->ne[0] = ne0;
    v->ne[1] = ne1;
    v->ne[2] = v->ne[3] = 1;
    v->type = t;
    if (t == Q_F32) {
        v->nb[3] = v->nb[2] = 4;
        v->nb[1] = 4;
        v->nb[0] = (size_t)ne1 * 4;
    } else {
        v->nb[0] = (size_t)(ne1 / 32) * 20;
        v->nb[1] = v->nb[2] = v->nb[3] = 20;
    }
    strncpy(v->name, name, sizeof v->name - 1);
    return v;
}

extern "C" {

q_error_code llama_build_graph(q_context* ctx, q_llama_model* model) {
    // validation order of upstream model.c:294-343
    if (!ctx || !model) return Q_ERR_NULL_PTR;
    if (!ctx->weights_mmap || !ctx->header) return Q_ERR_NULL_PTR;
    const q_model_header* h = ctx->header;
    if (h->magic != Q_MAGIC) return Q_ERR_INVALID_MAGIC;
    if (!h->n_layers || !h->dim || !h->vocab_size || !h->n_heads || !h->n_kv_heads)
        return Q_ERR_INVALID_CONFIG;
    if (h->dim % 32 || h->hidden_dim % 32) return Q_ERR_INVALID_CONFIG;
    if (h->dim % h->n_heads || h->n_heads % h->n_kv_heads || !h->hidden_dim || !h->max_seq_len)
        return Q_ERR_INVALID_CONFIG;
    q_llama_config& c = model->config;
    c.vocab_size = h->vocab_size;
    c.dim = h->dim;
    c.hidden_dim = h->hidden_dim;
    c.n_layers = h->n_layers;
    c.n_heads = h->n_heads;
    c.n_kv_heads = h->n_kv_heads;
    c.max_seq_len = h->max_seq_len;
    c.rope_freq_base = h->rope_freq_base;
    c.rms_norm_eps = (h->version >= 2 && h->rms_norm_eps > 0.0f) ? h->rms_norm_eps : 1e-5f;
    model->ctx = ctx;
    const uint32_t D = c.dim, H = c.hidden_dim, V = c.vocab_size;
    const uint32_t hd = D / c.n_heads, kvd = c.n_kv_heads * hd;
    size_t off = Q_HEADER_SIZE;
#define VIEW(dst, n0, n1, t, nm)                                             \
    do {                                                                     \
        size_t by = (t) == Q_F32 ? (size_t)(n0) * (n1) * 4                   \
                                 : (size_t)(n0) * ((n1) / 32) * 20;          \
        if (off + al64(by) > ctx->weights_size) return Q_ERR_INVALID_CONFIG; \
        dst = make_view(ctx, off, n0, n1, t, nm);                            \
        if (!dst) return Q_ERR_ARENA_OOM;                                    \
        off += al64(by);                                                     \
    } while (0)
    VIEW(model->token_embd, V, D, Q_F32, "token_embd.weight");
    VIEW(model->output_norm, D, 1, Q_F32, "output_norm.weight");
    VIEW(model->output, V, D, Q_F32, "output.weight");
    model->layers = (q_llama_layer*)q_arena_alloc(ctx, sizeof(q_llama_layer) * c.n_layers);
    if (!model->layers) return Q_ERR_ARENA_OOM;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        q_llama_layer* ly = &model->layers[l];
        memset(ly, 0, sizeof *ly);
        ly->layer_idx = l;
        VIEW(ly->attn_norm, D, 1, Q_F32, "attn_norm.weight");
        VIEW(ly->wq, D, D, Q_Q4_0, "wq.weight");
        VIEW(ly->wk, kvd, D, Q_Q4_0, "wk.weight");
        VIEW(ly->wv, kvd, D, Q_Q4_0, "wv.weight");
        VIEW(ly->wo, D, D, Q_Q4_0, "wo.weight");
        VIEW(ly->ffn_norm, D, 1, Q_F32, "ffn_norm.weight");
        VIEW(ly->w_gate, H, D, Q_Q4_0, "w_gate.weight");
        VIEW(ly->w_up, H, D, Q_Q4_0, "w_up.weight");
        VIEW(ly->w_down, D, H, Q_Q4_0, "w_down.weight");
    }
#undef VIEW
    // RoPE frequencies (+ host cos/sin cache when it fits, as upstream)
    const uint32_t np = hd / 2;
    model->rope_freqs = (float*)q_arena_alloc(ctx, np * sizeof(float));
    if (!model->rope_freqs) return Q_ERR_ARENA_OOM;
    for (uint32_t i = 0; i < np; ++i)
        model->rope_freqs[i] = powf(c.rope_freq_base, -2.0f * (float)i / (float)hd);
    model->rope_cache_enabled = false;
    model->rope_cos_cache = model->rope_sin_cache = nullptr;
    if (c.max_seq_len <= 8192) {
        const size_t cs = (size_t)c.max_seq_len * hd * sizeof(float);
        model->rope_cos_cache = (float*)q_arena_alloc(ctx, cs);
        model->rope_sin_cache = (float*)q_arena_alloc(ctx, cs);
        if (model->rope_cos_cache && model->rope_sin_cache) {
            for (uint32_t p = 0; p < c.max_seq_len; ++p)
                for (uint32_t i = 0; i < np; ++i) {
                    const float th = model->rope_freqs[i] * (float)p;
                    const size_t o = (size_t)p * hd + 2 * i;
                    model->rope_cos_cache[o] = model->rope_cos_cache[o + 1] = cosf(th);
                    model->rope_sin_cache[o] = model->rope_sin_cache[o + 1] = sinf(th);
                }
            model->rope_cache_enabled = true;
        }
    }
    ctx->scratch_base_offset = ctx->scratch_head;

    // one-time upload to HBM
    DevState* s = state_of(ctx, false);
    if (!s || !s->arena) return Q_ERR_INVALID_ARG;  // q_alloc_arena first (as upstream)
    q_error_code rc = upload_model(ctx, s, model);
    if (rc != Q_OK) return rc;
    if (ctx->kv_buffer) rc = ensure_graphs(ctx, s);
    return rc;
}

void llama_free_graph(q_llama_model* model) {
    if (!model) return;
    model->token_embd = model->output_norm = model->output = nullptr;
    model->layers = nullptr;
    model->ctx = nullptr;
    memset(&model->config, 0, sizeof model->config);
}

}  // extern "C"

static size_t kv_bytes_needed(const q_llama_config& c) {
    return (size_t)c.n_layers * c.n_kv_heads * c.max_seq_len * (c.dim / c.n_heads) * 2 * 4;
}

// Tensor-parallel ranks hold their vocab rows' logits; gather every rank's
// (ceil(V/W) rows each, in rank order) into logits_all.
static q_error_code gather_logits(DevState* s) {
    if (s->tp_world == 1) return Q_OK;
    if (s->peers_ready) {
        Q_CUDA(tp_allreduce(s, s->logits, s->tp.v_pad, TP_GATHER_F32, s->stream, s->logits_all));
        return Q_OK;
    }
    const NcclApi* n = nccl();
    if (!n) return Q_ERR_INVALID_ARG;
    const ncclResult_t r = n->all_gather(s->logits, s->logits_all, s->tp.v_pad, ncclFloat32, s->comm, s->stream);
    if (r != ncclSuccess) {
        set_last_error(n->error_string(r), cudaErrorUnknown);
        return Q_ERR_INVALID_ARG;
    }
    return Q_OK;
}

static q_error_code ready(q_llama_model* model, q_context* ctx, DevState** out) {
    DevState* s = state_of(ctx, false);
    if (!s || !s->built) return Q_ERR_INVALID_ARG;
    if (ctx->kv_size < kv_bytes_needed(model->config)) return Q_ERR_INVALID_ARG;
    q_error_code rc = ensure_graphs(ctx, s);
    if (rc != Q_OK) return rc;
    *out = s;
    return Q_OK;
}

// Prompts of more than one row take the tensor-core prefill path
// (csrc/prefill.cu; on tensor-parallel contexts every rank runs its shard and
// the partial residuals are all-reduced); QORUS_B200_PREFILL=0 forces the
// row replay below.
static bool use_prefill(const DevState* s, uint32_t seq_len) {
    if (seq_len < 2) return false;
    const char* e = std::getenv("QORUS_B200_PREFILL");
    return !(e && e[0] == '0');
}

// One graph replay per row: rows 0..seq_len-2 run the layer stack only, the
// last row also runs the LM head + argmax.  Row t sees the upstream softmax
// row length N = pos + seq_len and unmasked positions 0..pos+t.
static q_error_code run_rows(DevState* s, const uint32_t* tokens, uint32_t seq_len, uint32_t pos,
                             bool sample = false) {
    for (uint32_t t = 0; t < seq_len; ++t) {
        StepParams* hp = &s->h_step[t];
        hp->token = tokens[t];
        hp->pos = pos + t;
        hp->n_row = pos + seq_len;
        hp->valid = pos + t + 1;
        Q_CUDA(cudaMemcpyAsync(s->step, hp, sizeof *hp, cudaMemcpyHostToDevice, s->stream));
        const bool full = t + 1 == seq_len;
        Q_CUDA(cudaGraphLaunch(full ? (sample ? s->g_sample : s->g_full) : s->g_body, s->stream));
        g_kernel_launches.fetch_add(full ? s->kernels_full : s->kernels_body);
    }
    return Q_OK;
}

extern "C" {

q_error_code llama_forward(q_llama_model* model, q_context* ctx, const uint32_t* tokens,
                           uint32_t seq_len, uint32_t pos, float* logits) {
    // upstream model.c:1664-1685
    if (!model || !ctx || !tokens || !logits) return Q_ERR_INVALID_ARG;
    if (seq_len == 0) return Q_ERR_INVALID_SIZE;
    if (seq_len > model->config.max_seq_len) return Q_ERR_INVALID_SIZE;
    if (pos >= model->config.max_seq_len) return Q_ERR_INVALID_ARG;
    if (!ctx->scratch_buffer || !ctx->kv_buffer) return Q_ERR_INVALID_ARG;
    if ((uint64_t)pos + seq_len > model->config.max_seq_len) return Q_ERR_INVALID_ARG;
    for (uint32_t t = 0; t < seq_len; ++t)
        if (tokens[t] >= model->config.vocab_size) return Q_ERR_INVALID_ARG;
    DevState* s = nullptr;
    q_error_code rc = ready(model, ctx, &s);
    if (rc != Q_OK) return rc;
    Q_CUDA(cudaStreamSynchronize(s->stream));  // pinned step slots may still be in use
    if (use_prefill(s, seq_len))
        rc = run_prefill(s, (float*)ctx->kv_buffer, tokens, seq_len, pos);
    else
        rc = run_rows(s, tokens, seq_len, pos);
    if (rc != Q_OK) return rc;
    if ((rc = gather_logits(s)) != Q_OK) return rc;
    Q_CUDA(cudaMemcpyAsync(logits, s->tp_world > 1 ? s->logits_all : s->logits,
                           (size_t)model->config.vocab_size * 4, cudaMemcpyDeviceToHost, s->stream));
    Q_CUDA(cudaStreamSynchronize(s->stream));
    return check_device_status("llama_forward");
}

}  // extern "C"

// Upstream keeps one xorshift64* state per host thread, seeded 123456789
// (src/main.c:950-973); so does this library, and q_generate carries it to
// the device for its loop and back.
static thread_local unsigned long long t_rng_state = 123456789ULL;

namespace {
struct SampleOpWork {
    void* p = nullptr;
    size_t bytes = 0;
};
}  // namespace

extern "C" {

q_error_code q_sample_token(const float* logits, uint32_t vocab_size, float temperature,
                            uint32_t top_k, float top_p, uint32_t* token_id_out, q_context* ctx) {
    (void)ctx;
    if (!logits || !token_id_out) return Q_ERR_INVALID_ARG;
    if (vocab_size == 0) return Q_ERR_INVALID_SIZE;
    if (!(temperature >= 0.0f) || !std::isfinite(temperature)) return Q_ERR_INVALID_ARG;
    if (temperature < 1e-6f) {
        // upstream main.c:870-881 on the caller's host logits
        uint32_t bi = 0;
        float bv = logits[0];
        for (uint32_t i = 1; i < vocab_size; ++i)
            if (logits[i] > bv) {
                bv = logits[i];
                bi = i;
            }
        *token_id_out = bi;
        return Q_OK;
    }
    // temperature > 0: the device sampler on a copy of the caller's logits
    static std::mutex mu;
    static std::unordered_map<int, SampleOpWork> work;
    std::lock_guard<std::mutex> lk(mu);
    int dev = 0;
    Q_CUDA(cudaGetDevice(&dev));
    const size_t V = vocab_size, al = 256;
    const size_t o_probs = (V * 4 + al - 1) / al * al, o_keep = o_probs + (V * 4 + al - 1) / al * al;
    const size_t o_par = o_keep + (V + al - 1) / al * al, o_rng = o_par + al, o_key = o_rng + al, o_tok = o_key + al;
    const size_t need = o_tok + al;
    SampleOpWork& w = work[dev];
    if (w.bytes < need) {
        Q_CUDA(cudaDeviceSynchronize());
        if (w.p) cudaFree(w.p);
        w = SampleOpWork{};
        if (!cuda_ok(dev_malloc(&w.p, need), "dev_malloc(sampler)")) return Q_ERR_ALLOC_FAILED;
        w.bytes = need;
    }
    uint8_t* b = (uint8_t*)w.p;
    SampleParams prm{temperature, top_k, top_p, 0u};
    // upstream's vector temperature loop needs V >= 8 and 32-byte aligned logits
    prm.scalar_path = (vocab_size < 8 || ((uintptr_t)logits & 31)) ? 1u : 0u;
    cudaStream_t st = op_stream();
    Q_CUDA(cudaMemcpyAsync(b, logits, V * 4, cudaMemcpyHostToDevice, st));
    Q_CUDA(cudaMemcpyAsync(b + o_par, &prm, sizeof prm, cudaMemcpyHostToDevice, st));
    Q_CUDA(cudaMemcpyAsync(b + o_rng, &t_rng_state, 8, cudaMemcpyHostToDevice, st));
    SampleArgs sa{};
    sa.logits = (const float*)b;
    sa.V = vocab_size;
    sa.params = (const SampleParams*)(b + o_par);
    sa.rng = (unsigned long long*)(b + o_rng);
    sa.probs = (float*)(b + o_probs);
    sa.keep = b + o_keep;
    sa.best = (unsigned long long*)(b + o_key);
    sa.token_out = (uint32_t*)(b + o_tok);
    Q_CUDA(launch_ex(sample_kernel, dim3(1), dim3(SAMPLE_THREADS), 0, st, false, sa));
    uint32_t tok = 0;
    unsigned long long rs = 0;
    Q_CUDA(cudaMemcpyAsync(&tok, b + o_tok, 4, cudaMemcpyDeviceToHost, st));
    Q_CUDA(cudaMemcpyAsync(&rs, b + o_rng, 8, cudaMemcpyDeviceToHost, st));
    Q_CUDA(cudaStreamSynchronize(st));
    t_rng_state = rs;
    *token_id_out = tok;
    return Q_OK;
}

q_error_code q_generate(q_generation_state* st) {
    // upstream main.c:994-1131; the argmax is taken on the device
    if (!st || !st->ctx || !st->model || !st->tokenizer || !st->prompt_tokens ||
        !st->generated_tokens)
        return Q_ERR_INVALID_ARG;
    if (st->num_prompt_tokens == 0 || st->max_tokens == 0) return Q_ERR_INVALID_SIZE;
    if (!(st->temperature >= 0.0f) || !std::isfinite(st->temperature)) return Q_ERR_INVALID_ARG;
    if (!st->tokenizer->initialized) return Q_ERR_INVALID_ARG;
    if (!st->ctx->scratch_buffer || !st->ctx->kv_buffer) return Q_ERR_INVALID_ARG;
    const q_llama_config& c = st->model->config;
    if (st->num_prompt_tokens > c.max_seq_len) return Q_ERR_INVALID_SIZE;
    for (uint32_t t = 0; t < st->num_prompt_tokens; ++t)
        if (st->prompt_tokens[t] >= c.vocab_size) return Q_ERR_INVALID_ARG;
    st->num_generated_tokens = 0;
    st->current_pos = 0;
    q_arena_reset(st->ctx);
    DevState* s = nullptr;
    q_error_code rc = ready(st->model, st->ctx, &s);
    if (rc != Q_OK) return rc;
    Q_CUDA(cudaStreamSynchronize(s->stream));
    // temperature > 0: every token is drawn on the device by the sampler
    // (upstream q_sample_token per step, main.c:1044 and 1109) from this
    // thread's xorshift state, carried to the device and back
    const bool sample = st->temperature >= 1e-6f;
    if (sample) {
        if ((rc = ensure_sample_graph(st->ctx, s)) != Q_OK) return rc;
        const SampleParams prm{st->temperature, st->top_k, st->top_p, 0u};
        Q_CUDA(cudaMemcpy(s->samp, &prm, sizeof prm, cudaMemcpyHostToDevice));
        Q_CUDA(cudaMemcpy(s->rng, &t_rng_state, 8, cudaMemcpyHostToDevice));
    }
    // a forward is followed by a draw only when the loop below will take a
    // token from it (upstream draws inside the loop), so the thread's
    // random stream advances exactly as upstream's would
    const bool draw0 = sample && st->num_prompt_tokens < c.max_seq_len;
    if (use_prefill(s, st->num_prompt_tokens))
        rc = run_prefill(s, (float*)st->ctx->kv_buffer, st->prompt_tokens, st->num_prompt_tokens, 0, draw0);
    else
        rc = run_rows(s, st->prompt_tokens, st->num_prompt_tokens, 0, draw0);
    if (rc != Q_OK) return rc;
    st->current_pos = st->num_prompt_tokens;
    while (st->num_generated_tokens < st->max_tokens) {
        if (st->current_pos >= c.max_seq_len) break;
        uint32_t tok = 0;
        Q_CUDA(cudaMemcpyAsync(&tok, s->last_tok, 4, cudaMemcpyDeviceToHost, s->stream));
        Q_CUDA(cudaStreamSynchronize(s->stream));
        if ((rc = check_device_status("q_generate")) != Q_OK) return rc;
        if (tok >= c.vocab_size) return Q_ERR_INVALID_ARG;
        st->generated_tokens[st->num_generated_tokens++] = tok;
        if (tok == st->tokenizer->eos_token_id) break;
        q_arena_reset(st->ctx);
        const bool draw = sample && st->num_generated_tokens < st->max_tokens && st->current_pos + 1 < c.max_seq_len;
        if ((rc = run_rows(s, &tok, 1, st->current_pos, draw)) != Q_OK) return rc;
        st->current_pos++;
    }
    Q_CUDA(cudaStreamSynchronize(s->stream));
    if (sample) Q_CUDA(cudaMemcpy(&t_rng_state, s->rng, 8, cudaMemcpyDeviceToHost));
    return check_device_status("q_generate");
}

// ---- additive device-resident entry points -------------------------------------

void* q_b200_stream(q_context* ctx) {
    DevState* s = state_of(ctx, false);
    return s ? (void*)s->stream : nullptr;
}

const float* q_b200_device_logits(q_context* ctx) {
    DevState* s = state_of(ctx, false);
    return s ? (s->tp_world > 1 ? s->logits_all : s->logits) : nullptr;
}

q_error_code q_b200_kv_write(q_context* ctx, size_t off, const void* host, size_t bytes) {
    if (!ctx || !host || !ctx->kv_buffer) return Q_ERR_INVALID_ARG;
    if (off > ctx->kv_size || bytes > ctx->kv_size - off) return Q_ERR_INVALID_SIZE;
    if (DevState* s = state_of(ctx, false)) Q_CUDA(cudaStreamSynchronize(s->stream));
    Q_CUDA(cudaMemcpy((uint8_t*)ctx->kv_buffer + off, host, bytes, cudaMemcpyHostToDevice));
    return Q_OK;
}

q_error_code q_b200_kv_read(q_context* ctx, size_t off, void* host, size_t bytes) {
    if (!ctx || !host || !ctx->kv_buffer) return Q_ERR_INVALID_ARG;
    if (off > ctx->kv_size || bytes > ctx->kv_size - off) return Q_ERR_INVALID_SIZE;
    if (DevState* s = state_of(ctx, false)) Q_CUDA(cudaStreamSynchronize(s->stream));
    Q_CUDA(cudaMemcpy(host, (uint8_t*)ctx->kv_buffer + off, bytes, cudaMemcpyDeviceToHost));
    return Q_OK;
}

q_error_code q_b200_decode_loop(q_llama_model* model, q_context* ctx, uint32_t first_token,
                                uint32_t pos, uint32_t n_steps, uint32_t* out_tokens, int sync) {
    if (!model || !ctx) return Q_ERR_INVALID_ARG;
    if (n_steps == 0) return Q_ERR_INVALID_SIZE;
    if (first_token >= model->config.vocab_size) return Q_ERR_INVALID_ARG;
    if ((uint64_t)pos + n_steps > model->config.max_seq_len) return Q_ERR_INVALID_ARG;
    DevState* s = nullptr;
    q_error_code rc = ready(model, ctx, &s);
    if (rc != Q_OK) return rc;
    Q_CUDA(cudaStreamSynchronize(s->stream));  // h_step[0] may still be read by a prior copy
    StepParams* hp = &s->h_step[0];
    hp->token = first_token;
    hp->pos = pos;
    hp->n_row = hp->valid = pos + 1;
    Q_CUDA(cudaMemcpyAsync(s->step, hp, sizeof *hp, cudaMemcpyHostToDevice, s->stream));
    Q_CUDA(cudaMemsetAsync(s->tok_count, 0, 4, s->stream));
    for (uint32_t i = 0; i < n_steps; ++i) {
        Q_CUDA(cudaGraphLaunch(s->g_full, s->stream));
        g_kernel_launches.fetch_add(s->kernels_full);
    }
    if (!sync) return Q_OK;
    Q_CUDA(cudaStreamSynchronize(s->stream));
    if ((rc = check_device_status("q_b200_decode_loop")) != Q_OK) return rc;
    if (out_tokens) {
        const uint32_t n = std::min(n_steps, s->tok_cap);
        Q_CUDA(cudaMemcpy(out_tokens, s->tok_out, (size_t)n * 4, cudaMemcpyDeviceToHost));
    }
    return Q_OK;
}

q_error_code q_b200_profile_step(q_llama_model* model, q_context* ctx, uint32_t token,
                                 uint32_t pos, uint64_t* out, uint32_t max_kernels,
                                 uint32_t* n_kernels) {
    if (!model || !ctx || !out || !n_kernels) return Q_ERR_INVALID_ARG;
    if (token >= model->config.vocab_size || pos >= model->config.max_seq_len) return Q_ERR_INVALID_ARG;
    DevState* s = nullptr;
    q_error_code rc = ready(model, ctx, &s);
    if (rc != Q_OK) return rc;
    if ((rc = capture_trace_graph(ctx, s)) != Q_OK) return rc;
    std::vector<unsigned long long> buf((size_t)s->trace_slots * 4);
    for (size_t i = 0; i < s->trace_slots; ++i) {
        buf[4 * i] = buf[4 * i + 1] = ~0ull;
        buf[4 * i + 2] = buf[4 * i + 3] = 0ull;
    }
    Q_CUDA(cudaStreamSynchronize(s->stream));
    Q_CUDA(cudaMemcpy(s->trace_buf, buf.data(), buf.size() * 8, cudaMemcpyHostToDevice));
    StepParams* hp = &s->h_step[0];
    hp->token = token;
    hp->pos = pos;
    hp->n_row = hp->valid = pos + 1;
    Q_CUDA(cudaMemcpyAsync(s->step, hp, sizeof *hp, cudaMemcpyHostToDevice, s->stream));
    Q_CUDA(cudaMemsetAsync(s->tok_count, 0, 4, s->stream));
    Q_CUDA(cudaGraphLaunch(s->g_trace, s->stream));
    g_kernel_launches.fetch_add(s->kernels_full);
    Q_CUDA(cudaStreamSynchronize(s->stream));
    if ((rc = check_device_status("q_b200_profile_step")) != Q_OK) return rc;
    Q_CUDA(cudaMemcpy(buf.data(), s->trace_buf, buf.size() * 8, cudaMemcpyDeviceToHost));
    const uint32_t n = std::min(max_kernels, s->trace_slots);
    for (uint32_t i = 0; i < n; ++i)
        for (int k = 0; k < 3; ++k) out[3 * i + k] = buf[4 * i + k];
    *n_kernels = n;
    return Q_OK;
}

q_error_code q_b200_decode_greedy(q_llama_model* model, q_context* ctx, uint32_t token,
                                  uint32_t pos, uint32_t* next_token) {
    if (!next_token) return Q_ERR_INVALID_ARG;
    q_error_code rc = q_b200_decode_loop(model, ctx, token, pos, 1, nullptr, 1);
    if (rc != Q_OK) return rc;
    DevState* s = state_of(ctx, false);
    Q_CUDA(cudaMemcpy(next_token, s->last_tok, 4, cudaMemcpyDeviceToHost));
    return Q_OK;
}

}  // extern "C"
