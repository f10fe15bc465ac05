// model.cu — one-time model upload to HBM and the captured decode graphs.
//
// Upload (stands beside upstream llama_build_graph, model.c:294-673): every
// Q4_0 projection is repacked into stream tiles; wq|wk|wv become one matrix
// (one fused QKV launch), w_gate/w_up are row-interleaved (one fused
// gate-up-SiLU launch).  FP32 embedding / LM head / norms are copied as is.
// RoPE tables are built on the host exactly as upstream (powf/cosf/sinf in
// fp32, duplicated pairs, model.c:625-665) and uploaded.
//
// Per-token work (upstream llama_forward, model.c:1655-1850) is 6 kernels per
// layer — QKV(+RMSNorm, RoPE, KV store), attention scores, attention P.V +
// combine, wo(+residual), gate/up(+RMSNorm, SiLU*up), down(+residual) — plus
// the LM head(+final norm, argmax) and a step-advance kernel, captured once
// into CUDA graphs with programmatic dependent launch between kernels.
#include <cmath>
#include <cstdlib>

#include <cudaTypedefs.h>

#include "runtime.cuh"

namespace qb200 {

static q_error_code dalloc(DevState* s, void** p, size_t bytes) {
    if (!cuda_ok(dev_malloc(p, bytes ? bytes : 16), "dev_malloc(weights)")) return Q_ERR_ALLOC_FAILED;
    s->weight_allocs.push_back(*p);
    return Q_OK;
}

q_error_code upload_model(q_context* ctx, DevState* s, const q_llama_model* model) {
    (void)ctx;
    free_model(s);
    const q_llama_config& c = model->config;
    s->cfg = c;
    const uint32_t D = c.dim, H = c.hidden_dim, V = c.vocab_size, L = c.n_layers;
    s->hd = D / c.n_heads;
    s->kvd = c.n_kv_heads * s->hd;
    const uint32_t G = c.n_heads / c.n_kv_heads;
    if (!(s->hd == 32 || s->hd == 64 || s->hd == 128) || G > (uint32_t)ATT_MAXG ||
        c.n_heads % c.n_kv_heads || c.max_seq_len == 0 || D > GEMV_MAX_NORM_K || D % 4)
        return Q_ERR_INVALID_CONFIG;
    // this rank's shard (the whole model when tp_world == 1)
    if (!tp_shape(c, s->tp_rank, s->tp_world, s->tp)) return Q_ERR_INVALID_CONFIG;
    const TpShape& t = s->tp;
    if (!plan_gemv(t.d + 2 * t.kvd, D, s->p_qkv) || !plan_gemv(D, t.d, s->p_wo) ||
        !plan_gemv(2 * t.h, D, s->p_gu) || !plan_gemv(D, t.h, s->p_down))
        return Q_ERR_INVALID_CONFIG;
    // GEMV chains of a decode step: [qkv(0)], then per layer l after its
    // attention [wo(l), gate/up(l), down(l), qkv(l+1)] ([wo, gate/up, down]
    // for the last layer)
    {
        const GemvPlan* first[1] = {&s->p_qkv};
        const GemvPlan* mid[4] = {&s->p_wo, &s->p_gu, &s->p_down, &s->p_qkv};
        if (!plan_chain(first, 1, s->cp_first) || !plan_chain(mid, 4, s->cp_mid) ||
            !plan_chain(mid, 3, s->cp_last) || !plan_chain(&mid[0], 1, s->cp_wo) ||
            !plan_chain(&mid[1], 1, s->cp_gu) || !plan_chain(&mid[2], 1, s->cp_down))
            return Q_ERR_INVALID_CONFIG;
        // GEMVs per launch: 1 (separate kernels) unless QORUS_B200_CHAIN asks
        // for the persistent chain of a layer's GEMVs
        // (tensor-parallel ranks all-reduce between GEMVs: one per launch)
        const char* env = std::getenv("QORUS_B200_CHAIN");
        s->chain_phases = (env && env[0] == '1' && s->tp_world == 1) ? 4 : 1;
    }
    {
        const size_t sb = std::max(s->cp_first.scratch_bytes(),
                                   std::max(std::max(s->cp_mid.scratch_bytes(), s->cp_last.scratch_bytes()),
                 std::max(s->cp_wo.scratch_bytes(), std::max(s->cp_gu.scratch_bytes(), s->cp_down.scratch_bytes()))));
        void* sp = nullptr;
        q_error_code r = dalloc(s, &sp, sb);
        if (r != Q_OK) return r;
        if (!cuda_ok(cudaMemset(sp, 0, sb), "memset(gemv scratch)")) return Q_ERR_INVALID_ARG;
        s->gemv_scratch = sp;
        register_zero_area(sp, ChainPlan::kTicketWords * 4);
    }
    cudaStream_t st = s->stream;
    const size_t nbD = D / 32, nbH = H / 32;
    const size_t qkv_aos = (size_t)(t.d + 2 * t.kvd) * nbD * 20;
    const size_t gu_aos = (size_t)2 * t.h * nbD * 20;
    const size_t down_aos = (size_t)D * (t.h / 32) * 20;
    const size_t stage_bytes = std::max(qkv_aos, std::max(gu_aos, down_aos));
    uint8_t* stage = nullptr;
    if (!cuda_ok(dev_malloc(&stage, stage_bytes), "dev_malloc(stage)")) return Q_ERR_ALLOC_FAILED;
    q_error_code rc = Q_OK;
    auto h2d = [&](void* dst, const void* src, size_t n) {
        return cuda_ok(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, st), "upload");
    };
    // Rows of a Q4_0 matrix are contiguous AoS blocks; a K-slice (wo, down
    // under tensor parallelism) is gathered row by row on the host first.
    std::vector<uint8_t> hcols;
    auto kslice = [&](const q_tensor* w, uint32_t rows, uint32_t nb_full, uint32_t blk0,
                      uint32_t nblk) -> const void* {
        if (nblk == nb_full) return w->data;
        hcols.resize((size_t)rows * nblk * 20);
        const uint8_t* src = (const uint8_t*)w->data;
        for (uint32_t r = 0; r < rows; ++r)
            std::memcpy(hcols.data() + (size_t)r * nblk * 20, src + ((size_t)r * nb_full + blk0) * 20,
                        (size_t)nblk * 20);
        return hcols.data();
    };
    const size_t rowD = (size_t)nbD * 20;  // bytes of one row with K = D
    void* p = nullptr;
    for (uint32_t l = 0; l < L && rc == Q_OK; ++l) {
        const q_llama_layer& ly = model->layers[l];
        if ((rc = dalloc(s, &p, s->p_qkv.packed_bytes))) break;
        s->qkv.push_back((uint8_t*)p);
        if (!h2d(stage, (const uint8_t*)ly.wq->data + t.q0 * rowD, t.d * rowD) ||
            !h2d(stage + t.d * rowD, (const uint8_t*)ly.wk->data + t.kv0 * rowD, t.kvd * rowD) ||
            !h2d(stage + (t.d + t.kvd) * rowD, (const uint8_t*)ly.wv->data + t.kv0 * rowD, t.kvd * rowD) ||
            !cuda_ok(pack_q4(stage, s->p_qkv, 0, s->qkv.back(), st), "pack qkv")) {
            rc = Q_ERR_INVALID_ARG;
            break;
        }
        if ((rc = dalloc(s, &p, s->p_wo.packed_bytes))) break;
        s->wo.push_back((uint8_t*)p);
        if (!h2d(stage, kslice(ly.wo, D, nbD, t.q0 / 32, t.d / 32), (size_t)D * (t.d / 32) * 20) ||
            !cuda_ok(pack_q4(stage, s->p_wo, 0, s->wo.back(), st), "pack wo")) {
            rc = Q_ERR_INVALID_ARG;
            break;
        }
        if ((rc = dalloc(s, &p, s->p_gu.packed_bytes))) break;
        s->gu.push_back((uint8_t*)p);
        if (!h2d(stage, (const uint8_t*)ly.w_gate->data + t.h0 * rowD, t.h * rowD) ||
            !h2d(stage + t.h * rowD, (const uint8_t*)ly.w_up->data + t.h0 * rowD, t.h * rowD) ||
            !cuda_ok(pack_q4(stage, s->p_gu, t.h, s->gu.back(), st), "pack gate/up")) {
            rc = Q_ERR_INVALID_ARG;
            break;
        }
        if ((rc = dalloc(s, &p, s->p_down.packed_bytes))) break;
        s->down.push_back((uint8_t*)p);
        if (!h2d(stage, kslice(ly.w_down, D, nbH, t.h0 / 32, t.h / 32), down_aos) ||
            !cuda_ok(pack_q4(stage, s->p_down, 0, s->down.back(), st), "pack down")) {
            rc = Q_ERR_INVALID_ARG;
            break;
        }
    }
    if (rc == Q_OK) {
        rc = dalloc(s, &p, (size_t)L * D * 4);
        s->attn_norm = (float*)p;
    }
    if (rc == Q_OK) {
        rc = dalloc(s, &p, (size_t)L * D * 4);
        s->ffn_norm = (float*)p;
    }
    for (uint32_t l = 0; l < L && rc == Q_OK; ++l)
        if (!h2d(s->attn_norm + (size_t)l * D, model->layers[l].attn_norm->data, (size_t)D * 4) ||
            !h2d(s->ffn_norm + (size_t)l * D, model->layers[l].ffn_norm->data, (size_t)D * 4))
            rc = Q_ERR_INVALID_ARG;
    if (rc == Q_OK && !(rc = dalloc(s, &p, (size_t)D * 4))) {
        s->out_norm = (float*)p;
        if (!h2d(p, model->output_norm->data, (size_t)D * 4)) rc = Q_ERR_INVALID_ARG;
    }
    if (rc == Q_OK && !(rc = dalloc(s, &p, (size_t)V * D * 4))) {
        s->embd = (float*)p;
        if (!h2d(p, model->token_embd->data, (size_t)V * D * 4)) rc = Q_ERR_INVALID_ARG;
    }
    if (rc == Q_OK && !(rc = dalloc(s, &p, (size_t)t.v * D * 4))) {  // this rank's vocab rows
        s->out_w = (float*)p;
        if (!h2d(p, (const float*)model->output->data + (size_t)t.v0 * D, (size_t)t.v * D * 4))
            rc = Q_ERR_INVALID_ARG;
    }
    if (rc == Q_OK && s->tp_world > 1 && !(rc = dalloc(s, &p, (size_t)s->tp_world * t.v_pad * 4)))
        s->logits_all = (float*)p;
    // RoPE tables, host-built like upstream model.c:625-665
    const size_t tab = (size_t)c.max_seq_len * s->hd;
    std::vector<float> ct(tab), stb(tab);
    {
        const uint32_t np = s->hd / 2;
        std::vector<float> fr(np);
        for (uint32_t i = 0; i < np; ++i) fr[i] = powf(c.rope_freq_base, -2.0f * (float)i / (float)s->hd);
        for (uint32_t ps = 0; ps < c.max_seq_len; ++ps)
            for (uint32_t i = 0; i < np; ++i) {
                const float th = fr[i] * (float)ps;
                const float cv = cosf(th), sv = sinf(th);
                const size_t o = (size_t)ps * s->hd + 2 * i;
                ct[o] = ct[o + 1] = cv;
                stb[o] = stb[o + 1] = sv;
            }
    }
    if (rc == Q_OK && !(rc = dalloc(s, &p, tab * 4))) {
        s->rope_cos = (float*)p;
        if (!h2d(p, ct.data(), tab * 4)) rc = Q_ERR_INVALID_ARG;
    }
    if (rc == Q_OK && !(rc = dalloc(s, &p, tab * 4))) {
        s->rope_sin = (float*)p;
        if (!h2d(p, stb.data(), tab * 4)) rc = Q_ERR_INVALID_ARG;
    }
    if (rc == Q_OK && !cuda_ok(cudaStreamSynchronize(st), "upload sync")) rc = Q_ERR_INVALID_ARG;
    cudaFree(stage);
    if (rc != Q_OK) {
        free_model(s);
        return rc;
    }

    // activations: carved from the device arena once; the watermark moves
    // past them so per-token work allocates nothing
    s->arena_head = 0;
    if ((rc = plan_attention(s)) != Q_OK) {
        free_model(s);
        return rc;
    }
    s->tok_cap = c.max_seq_len;
    s->x = (float*)dev_arena_alloc(s, (size_t)D * 4);
    s->q = (float*)dev_arena_alloc(s, (size_t)D * 4);
    s->att = (float*)dev_arena_alloc(s, (size_t)D * 4);
    s->h = (float*)dev_arena_alloc(s, (size_t)H * 4);
    s->logits = (float*)dev_arena_alloc(s, (size_t)V * 4);
    s->chain_bar = (uint32_t*)dev_arena_alloc(s, (size_t)L * GEMV_MAX_PHASES * 4);
    s->best = (unsigned long long*)dev_arena_alloc(s, 8);
    s->step = (StepParams*)dev_arena_alloc(s, sizeof(StepParams));
    s->tok_out = (uint32_t*)dev_arena_alloc(s, (size_t)s->tok_cap * 4);
    s->tok_count = (uint32_t*)dev_arena_alloc(s, 4);
    s->last_tok = (uint32_t*)dev_arena_alloc(s, 4);
    s->samp = (SampleParams*)dev_arena_alloc(s, sizeof(SampleParams));
    s->rng = (unsigned long long*)dev_arena_alloc(s, 8);
    if (!s->x || !s->q || !s->att || !s->h || !s->logits || !s->best || !s->step || !s->tok_out ||
        !s->tok_count || !s->last_tok || !s->chain_bar || !s->samp || !s->rng) {
        free_model(s);
        return Q_ERR_ARENA_OOM;
    }
    s->arena_base = s->arena_head;
    register_zero_area(s->chain_bar, (size_t)L * GEMV_MAX_PHASES * 4);
    if (!cuda_ok(cudaMemsetAsync(s->best, 0, 8, st), "init") ||
        !cuda_ok(cudaMemsetAsync(s->chain_bar, 0, (size_t)L * GEMV_MAX_PHASES * 4, st), "init") ||
        !cuda_ok(cudaMemsetAsync(s->tok_count, 0, 4, st), "init") ||
        !cuda_ok(cudaStreamSynchronize(st), "init sync")) {
        free_model(s);
        return Q_ERR_INVALID_ARG;
    }
    if (s->h_step) cudaFreeHost(s->h_step);
    s->h_step = nullptr;
    if (!cuda_ok(cudaMallocHost(&s->h_step, sizeof(StepParams) * (size_t)c.max_seq_len), "pinned")) {
        free_model(s);
        return Q_ERR_ALLOC_FAILED;
    }
    s->built = true;
    return Q_OK;
}

// ---- graph capture ------------------------------------------------------------------

// Next step-trace slot while capturing the traced graph, else null.
static unsigned long long* take_slot(DevState* s) {
    if (!s->tr_next) return nullptr;
    unsigned long long* p = s->tr_next;
    s->tr_next += 4;
    return p;
}

// The attention instantiation for (head_dim, query heads per KV head).
template <int HD>
static const void* attn_kernel_g(uint32_t G) {
    switch (G) {
        case 1: return (const void*)attn_decode_kernel<HD, 1>;
        case 2: return (const void*)attn_decode_kernel<HD, 2>;
        case 4: return (const void*)attn_decode_kernel<HD, 4>;
        case 8: return (const void*)attn_decode_kernel<HD, 8>;
        default: return nullptr;
    }
}

static const void* attn_kernel_for(uint32_t hd, uint32_t G) {
    switch (hd) {
        case 32: return attn_kernel_g<32>(G);
        case 64: return attn_kernel_g<64>(G);
        case 128: return attn_kernel_g<128>(G);
        default: return nullptr;
    }
}

// Attention launch shape: the largest cluster (16, else 8, 4, 2) and the
// deepest ring (<= 8 slots of 16 KB) with which all n_kv clusters are
// resident at once (one wave).
q_error_code plan_attention(DevState* s) {
    const q_llama_config& c = s->cfg;
    const uint32_t G = c.n_heads / c.n_kv_heads;
    const void* kern = attn_kernel_for(s->hd, G);
    if (!kern || G == 0 || G > (uint32_t)ATT_MAXG) return Q_ERR_INVALID_CONFIG;
    const size_t limit = 227 * 1024 - 8 * 1024;  // dynamic shared memory beside the static part
    for (uint32_t cs = 16; cs >= 2; cs /= 2) {
        if (cs > 8 &&
            cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        // chunks are whole ring stages of sp rows (the kernel's split)
        const uint32_t sp = ATT_STAGE_BYTES / (s->hd * 4);
        const uint32_t ca = ((c.max_seq_len + sp - 1) / sp + cs - 1) / cs * sp;
        for (uint32_t slots = ATT_MAX_SLOTS; slots >= 2; --slots) {
            const size_t smem = attn_smem_bytes(G, s->hd, ca, slots);
            if (smem > limit) continue;
            if (!cuda_ok(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                         "attention smem attribute"))
                return Q_ERR_INVALID_ARG;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(cs, s->tp.nkv);
            cfg.blockDim = dim3(ATT_THREADS);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = cs;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
                cudaGetLastError();
                continue;
            }
            if (n < (int)s->tp.nkv && !(cs == 2 && slots == 2 && n >= 1)) continue;
            s->att_cs = cs;
            s->att_ca = ca;
            s->att_slots = slots;
            s->att_smem = smem;
            return Q_OK;
        }
    }
    set_last_error("plan_attention: no cluster shape fits", cudaErrorInvalidConfiguration);
    return Q_ERR_INVALID_CONFIG;
}

// 3-D tensor map over the whole KV cache: x = the 2*hd floats of a position
// (K then V), y = position, z = layer * n_kv + kv head.  Boxes of
// ATT_STAGE_BYTES: hd floats by ATT_STAGE_BYTES / (4 hd) positions.
PFN_cuTensorMapEncodeTiled tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
    });
    if (!encode) set_last_error("cuTensorMapEncodeTiled unavailable", cudaErrorNotSupported);
    return encode;
}

static q_error_code make_kv_map(DevState* s, void* kv) {
    const PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
    if (!encode) return Q_ERR_INVALID_ARG;
    const q_llama_config& c = s->cfg;
    const uint32_t hd = s->hd;
    // (a tensor-parallel rank's cache holds its own KV heads only)
    const cuuint64_t dims[3] = {2ull * hd, c.max_seq_len, (cuuint64_t)c.n_layers * s->tp.nkv};
    const cuuint64_t strides[2] = {2ull * hd * 4, 2ull * hd * 4 * c.max_seq_len};
    const cuuint32_t box[3] = {hd, ATT_STAGE_BYTES / (4 * hd), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode(&s->kv_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, kv, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_last_error("cuTensorMapEncodeTiled(kv cache)", cudaErrorInvalidValue);
        return Q_ERR_INVALID_ARG;
    }
    return Q_OK;
}

static cudaError_t enqueue_attention(DevState* s, uint32_t layer, cudaStream_t st) {
    AttnArgs a{};
    a.q = s->q;
    a.layer = layer;
    a.trace = take_slot(s);
    a.out = s->att;
    a.step = s->step;
    a.n_heads = s->tp.nh;
    a.n_kv_heads = s->tp.nkv;
    a.max_seq = s->cfg.max_seq_len;
    a.chunk_alloc = s->att_ca;
    a.slots = s->att_slots;
    a.scale = 1.0f / sqrtf((float)s->hd);  // upstream model.c:1315
    // one cluster per KV head; programmatic overlap with the QKV GEMV before
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s->att_cs, s->tp.nkv);
    cfg.blockDim = dim3(ATT_THREADS);
    cfg.dynamicSmemBytes = s->att_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = s->att_cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    const void* kern = attn_kernel_for(s->hd, s->cfg.n_heads / s->cfg.n_kv_heads);
    if (!kern) return cudaErrorInvalidValue;
    void* params[2] = {&a, &s->kv_map};
    return cudaLaunchKernelExC(&cfg, kern, params);
}

// QKV projection of layer l (RMSNorm prologue; RoPE, KV store epilogue);
// layer 0 gathers the embedding row and keeps a copy as the residual stream.
static GemvArgs qkv_args(DevState* s, float* kv, uint32_t l) {
    const q_llama_config& c = s->cfg;
    const size_t layer_floats = (size_t)s->tp.nkv * c.max_seq_len * 2 * s->hd;
    GemvArgs g{};
    g.w = s->qkv[l];
    g.step = s->step;
    g.gather = l == 0;
    g.x = l == 0 ? s->embd : s->x;
    g.x_copy = l == 0 ? s->x : nullptr;
    g.norm_w = s->attn_norm + (size_t)l * c.dim;
    g.eps = c.rms_norm_eps;
    g.y = s->q;
    g.epi = EPI_QKV;
    g.rope_cos = s->rope_cos;
    g.rope_sin = s->rope_sin;
    g.kv_layer = kv + (size_t)l * layer_floats;
    g.hd = s->hd;
    g.q_rows = s->tp.d;
    g.kv_rows = s->tp.kvd;
    g.max_seq = c.max_seq_len;
    return g;
}

// The residual update of wo / down: y = x + W v, except on tensor-parallel
// ranks other than 0, which store their partial W v alone (the all-reduce
// that follows adds the partials and rank 0's x).
static int residual_epi(const DevState* s) {
    return s->tp_world > 1 && s->tp_rank != 0 ? EPI_STORE : EPI_RESID;
}

static cudaError_t nccl_status(ncclResult_t r) {
    if (r == ncclSuccess) return cudaSuccess;
    const NcclApi* n = nccl();
    set_last_error(n ? n->error_string(r) : "nccl", cudaErrorUnknown);
    return cudaErrorUnknown;
}

// In-place sum of `count` floats over the tensor-parallel ranks (no-op alone).
static cudaError_t allreduce_sum(DevState* s, float* buf, size_t count, cudaStream_t st) {
    if (s->tp_world == 1) return cudaSuccess;
    if (s->peers_ready) return tp_allreduce(s, buf, (uint32_t)count, TP_SUM_F32, st);
    const NcclApi* n = nccl();
    if (!n) return cudaErrorUnknown;
    return nccl_status(n->all_reduce(buf, buf, count, ncclFloat32, ncclSum, s->comm, st));
}

// Tensor-parallel exchange fused into the GEMVs (peer memory only; set
// QORUS_B200_TP_FUSED=0 for the separate all-reduce kernel): wo and down
// send their rows to every rank, gate/up and the next layer's QKV receive
// and sum them.  Parity 0 carries wo's exchange, parity 1 down's.
static bool tp_fused(const DevState* s) {
    if (s->tp_world < 2 || !s->peers_ready) return false;
    const char* e = getenv("QORUS_B200_TP_FUSED");
    return !(e && e[0] == '0');
}
static void tp_geometry(const DevState* s, GemvTp& t) {
    for (uint32_t r = 0; r < s->tp_world; ++r) t.tp_base[r] = s->peers.base[r];
    t.tp_off = (uint32_t)tp_fused_offset(s->tp_world, s->peer_slice);
    t.tp_slice = s->peer_slice;
    t.tp_world = s->tp_world;
    t.tp_rank = s->tp_rank;
}
static void tp_fuse(const DevState* s, GemvArgs& g, GemvTp& t, bool send, uint32_t par) {
    tp_geometry(s, t);
    t.tp_par = par;
    if (send) {
        t.tp_send = 1;
    } else {
        t.tp_recv = 1;
        g.x_copy = s->x;  // CTA 0 stores the summed input: the residual stream
    }
}

// head_recv: the LM head follows and takes the last layer's down exchange
// itself (fused tensor-parallel exchange only).
static cudaError_t enqueue_layers(DevState* s, float* kv, cudaStream_t st, bool head_recv = false) {
    const q_llama_config& c = s->cfg;
    const uint32_t D = c.dim;
    GemvArgs first = qkv_args(s, kv, 0);
    const GemvPlan* fm[1] = {&s->p_qkv};
    cudaError_t e = launch_chain(s->cp_first, fm, &first, s->gemv_scratch, nullptr, take_slot(s), st, false);
    for (uint32_t l = 0; l < c.n_layers && e == cudaSuccess; ++l) {
        e = enqueue_attention(s, l, st);
        if (e != cudaSuccess) break;
        GemvArgs ph[4] = {};
        ph[0].w = s->wo[l];  // attention output -> residual
        ph[0].step = s->step;
        ph[0].x = s->att;
        ph[0].y = s->x;
        ph[0].resid = s->x;
        ph[0].epi = residual_epi(s);
        ph[1].w = s->gu[l];  // RMSNorm -> gate/up -> SiLU(gate) * up
        ph[1].step = s->step;
        ph[1].x = s->x;
        ph[1].norm_w = s->ffn_norm + (size_t)l * D;
        ph[1].eps = c.rms_norm_eps;
        ph[1].y = s->h;
        ph[1].epi = EPI_SILU;
        ph[2].w = s->down[l];  // down -> residual
        ph[2].step = s->step;
        ph[2].x = s->h;
        ph[2].y = s->x;
        ph[2].resid = s->x;
        ph[2].epi = residual_epi(s);
        const bool more = l + 1 < c.n_layers;
        if (more) ph[3] = qkv_args(s, kv, l + 1);
        GemvTp tps[4] = {};
        if (tp_fused(s)) {
            tp_fuse(s, ph[0], tps[0], true, 0);
            tp_fuse(s, ph[1], tps[1], false, 0);
            // the last layer's down feeds the LM head's prologue, or (rows
            // without a head) the all-reduce kernel
            if (more || head_recv) tp_fuse(s, ph[2], tps[2], true, 1);
            if (more) tp_fuse(s, ph[3], tps[3], false, 1);
        }
        const GemvPlan* mats[4] = {&s->p_wo, &s->p_gu, &s->p_down, &s->p_qkv};
        if (s->chain_phases > 1) {
            e = launch_chain(more ? s->cp_mid : s->cp_last, mats, ph, s->gemv_scratch,
                             s->chain_bar + (size_t)l * GEMV_MAX_PHASES, take_slot(s), st, true);
        } else {
            // one GEMV per launch, chained by programmatic dependent launch
            const ChainPlan* one[4] = {&s->cp_wo, &s->cp_gu, &s->cp_down, &s->cp_first};
            for (uint32_t i = 0; i < (more ? 4u : 3u) && e == cudaSuccess; ++i) {
                e = launch_chain(*one[i], &mats[i], &ph[i], s->gemv_scratch, nullptr, take_slot(s), st, true,
                                 &tps[i]);
                // wo and down hold partial residual updates on a tensor-parallel rank
                if (e == cudaSuccess && (i == 0 || i == 2) && !tps[i].tp_send) e = allreduce_sum(s, s->x, c.dim, st);
            }
        }
    }
    return e;
}

// LM head (+ final norm, argmax) over residual row x (default: the decode
// residual stream), optionally the sampler (which replaces the argmax key
// with a drawn token when the context's temperature is above 0), then the
// step advance.
static cudaError_t enqueue_head(DevState* s, cudaStream_t st, const float* x = nullptr, bool sample = false,
                                bool tp_recv = false) {
    HeadArgs h{};
    const bool fused = tp_fused(s);
    if (fused) {  // argmax keys over peer memory; the receive of the last down exchange if asked
        tp_geometry(s, h.tp);
        h.tp_key = sample ? 0u : 1u;  // a sampled token comes from the gathered logits instead
        if (tp_recv) {
            h.tp.tp_recv = 1;
            h.tp.tp_par = 1;
            h.x_copy = s->x;
        }
    }
    h.w = s->out_w;
    h.x = x ? x : s->x;
    h.norm_w = s->out_norm;
    h.eps = s->cfg.rms_norm_eps;
    h.rows = s->tp.v;
    h.K = s->cfg.dim;
    h.row_base = s->tp.v0;
    h.logits = s->logits;
    h.best = s->best;
    h.trace = take_slot(s);
    h.slots = head_slots(h.K);
    if (!h.slots) return cudaErrorInvalidValue;
    {
        const cudaError_t e = ensure_smem_attr((const void*)lm_head_kernel, 227 * 1024);
        if (e != cudaSuccess) return e;
    }
    // one CTA per SM, each a contiguous range of rows
    const uint32_t grid = std::max<uint32_t>(1, std::min<uint32_t>(device_sms(), s->tp.v));
    const size_t smem = head_smem_bytes(h.K, h.slots);
    cudaError_t e = launch_ex(lm_head_kernel, dim3(grid), dim3(HEAD_THREADS), smem, st, true, h);
    if (e != cudaSuccess) return e;
    if (fused) {
        // advance_kernel reduces the keys
    } else if (s->tp_world > 1 && s->peers_ready) {  // the argmax key over every rank's vocab rows
        e = tp_allreduce(s, s->best, 1, TP_MAX_U64, st);
        if (e != cudaSuccess) return e;
    } else if (s->tp_world > 1) {
        const NcclApi* n = nccl();
        if (!n) return cudaErrorUnknown;
        e = nccl_status(n->all_reduce(s->best, s->best, 1, ncclUint64, ncclMax, s->comm, st));
        if (e != cudaSuccess) return e;
    }
    if (sample) {
        // the sampler needs the whole vocabulary: on a tensor-parallel
        // context every rank gathers all ranks' rows (rank order = vocabulary
        // order) and draws the same token from the same random state
        if (s->tp_world > 1) {
            if (s->peers_ready) {
                e = tp_allreduce(s, s->logits, s->tp.v_pad, TP_GATHER_F32, st, s->logits_all);
            } else {
                const NcclApi* n = nccl();
                if (!n) return cudaErrorUnknown;
                e = nccl_status(n->all_gather(s->logits, s->logits_all, s->tp.v_pad, ncclFloat32, s->comm, st));
            }
            if (e != cudaSuccess) return e;
        }
        SampleArgs sa{};
        sa.logits = s->tp_world > 1 ? s->logits_all : s->logits;
        sa.V = s->cfg.vocab_size;
        sa.params = s->samp;
        sa.rng = s->rng;
        sa.probs = s->samp_probs;
        sa.keep = s->samp_keep;
        sa.best = s->best;
        e = launch_ex(sample_kernel, dim3(1), dim3(SAMPLE_THREADS), 0, st, true, sa);
        if (e != cudaSuccess) return e;
    }
    AdvanceArgs a{};
    a.step = s->step;
    a.best = s->best;
    a.token_out = s->tok_out;
    a.token_count = s->tok_count;
    a.token_cap = s->tok_cap;
    a.last_token = s->last_tok;
    a.trace = take_slot(s);
    if (fused && !sample) {
        a.key_ctl = reinterpret_cast<uint32_t*>(s->peers.base[s->tp_rank] + h.tp.tp_off +
                                                (size_t)2 * s->tp_world * s->peer_slice * 8);
        a.key_world = s->tp_world;
    }
    return launch_ex(advance_kernel, dim3(1), dim3(32), 0, st, true, a);
}

static q_error_code capture(DevState* s, float* kv, bool with_head, cudaGraphExec_t* out,
                            uint64_t* n_kernels, bool sample = false) {
    cudaStream_t st = s->stream;
    cudaGraph_t g = nullptr;
    const uint64_t before = g_kernel_launches.load();
    if (!cuda_ok(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture"))
        return Q_ERR_INVALID_ARG;
    const bool head_recv = with_head && tp_fused(s);
    cudaError_t e = enqueue_layers(s, kv, st, head_recv);
    if (e == cudaSuccess && with_head) e = enqueue_head(s, st, nullptr, sample, head_recv);
    cudaError_t e2 = cudaStreamEndCapture(st, &g);
    *n_kernels = g_kernel_launches.load() - before;
    g_kernel_launches.fetch_sub(*n_kernels);  // captured, not launched
    if (!cuda_ok(e, "capture launches") || !cuda_ok(e2, "end capture")) {
        if (g) cudaGraphDestroy(g);
        return Q_ERR_INVALID_ARG;
    }
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return cuda_ok(e, "graph instantiate") ? Q_OK : Q_ERR_INVALID_ARG;
}

q_error_code capture_trace_graph(q_context* ctx, DevState* s) {
    if (s->g_trace) return Q_OK;
    const uint32_t slots = s->cfg.n_layers * 6 + 4;
    if (!s->trace_buf &&
        !cuda_ok(dev_malloc(&s->trace_buf, (size_t)slots * 4 * sizeof(unsigned long long)), "trace buf"))
        return Q_ERR_ALLOC_FAILED;
    s->trace_slots = slots;
    s->tr_next = s->trace_buf;
    uint64_t nk = 0;
    q_error_code rc = capture(s, (float*)ctx->kv_buffer, true, &s->g_trace, &nk);
    s->trace_slots = (uint32_t)((s->tr_next - s->trace_buf) / 4);
    s->tr_next = nullptr;
    return rc;
}

// The sampler's scratch ([V] probabilities and keep flags) is allocated on
// the first sampled generation, not at build time, so greedy-only callers
// never pay for it.
q_error_code ensure_sample_scratch(DevState* s) {
    if (s->samp_probs) return Q_OK;
    const size_t V = s->cfg.vocab_size;
    void* p = nullptr;
    if (!cuda_ok(dev_malloc(&p, V * 5 + 256), "dev_malloc(sampler scratch)")) return Q_ERR_ALLOC_FAILED;
    s->samp_probs = (float*)p;
    s->samp_keep = (uint8_t*)p + (V * 4 + 255) / 256 * 256;
    return Q_OK;
}

q_error_code ensure_sample_graph(q_context* ctx, DevState* s) {
    if (s->g_sample) return Q_OK;
    q_error_code rc = ensure_sample_scratch(s);
    if (rc != Q_OK) return rc;
    uint64_t nk = 0;
    return capture(s, (float*)ctx->kv_buffer, true, &s->g_sample, &nk, true);
}

q_error_code ensure_graphs(q_context* ctx, DevState* s) {
    if (s->g_full && s->graph_kv == ctx->kv_buffer) return Q_OK;
    if (s->g_body) cudaGraphExecDestroy(s->g_body);
    if (s->g_full) cudaGraphExecDestroy(s->g_full);
    if (s->g_trace) cudaGraphExecDestroy(s->g_trace);
    if (s->g_sample) cudaGraphExecDestroy(s->g_sample);
    s->g_body = s->g_full = s->g_trace = s->g_sample = nullptr;
    float* kv = (float*)ctx->kv_buffer;
    q_error_code rc = make_kv_map(s, kv);
    if (rc == Q_OK) rc = capture(s, kv, false, &s->g_body, &s->kernels_body);
    if (rc == Q_OK) rc = capture(s, kv, true, &s->g_full, &s->kernels_full);
    if (rc == Q_OK) s->graph_kv = ctx->kv_buffer;
    return rc;
}

}  // namespace qb200
