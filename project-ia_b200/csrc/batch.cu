// batch.cu — host side of batched decode (kernels in batch.cuh) and its
// additive entry points (include/qorus_b200.h).
//
// One step of B sequences, captured once into a CUDA graph:
//   per layer: inputs -> fragments (RMSNorm) -> QKV (RoPE, each sequence's
//   KV store at its own position) -> attention (grid z = sequence) ->
//   fragments -> wo (+ residual) -> fragments (RMSNorm) -> gate/up (SiLU*up)
//   -> fragments -> down (+ residual);
//   then fragments (final RMSNorm) -> LM head for all B rows (argmax keys)
//   -> advance (every sequence's token and position).
// Per-sequence step scalars live in device memory, so the graph replays
// for any positions; the argmax is fed back on the device.
#include "runtime.cuh"

namespace qb200 {

static size_t bal(size_t n) { return (n + 255) & ~(size_t)255; }

void free_batch(DevState* s) {
    BatchState& b = s->batch;
    if (b.graph) cudaGraphExecDestroy(b.graph);
    if (b.base) cudaFree(b.base);
    if (b.kv) cudaFree(b.kv);
    if (b.gath) cudaFree(b.gath);
    if (b.d_pages) cudaFree(b.d_pages);
    if (b.h_step) cudaFreeHost(b.h_step);
    b = BatchState{};
}

__global__ void absmax_kernel(const float* __restrict__ x, size_t n, uint32_t* out) {
    float m = 0.0f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

static cudaError_t launch_xprep(DevState* s, const BatchPrepArgs& a, cudaStream_t st) {
    cudaError_t e = ensure_smem_attr((const void*)batch_xprep_kernel, 227 * 1024);
    if (e != cudaSuccess) return e;
    if ((size_t)a.K * 4 > 220 * 1024) return cudaErrorInvalidValue;
    (void)s;
    // slices: enough CTAs that the conversion is not left to 8-16 SMs
    const uint32_t slices = std::max<uint32_t>(1, std::min<uint32_t>(a.K / 256, 128 / (a.TG * 8)));
    return launch_ex(batch_xprep_kernel, dim3(a.TG * 8, slices), dim3(256), (size_t)a.K * 4, st, true, a);
}

static cudaError_t launch_bgemv(DevState* s, const uint8_t* w, const GemvPlan& p, BatchGemvArgs a, cudaStream_t st) {
    const BatchState& b = s->batch;
    a.w = w;
    a.M = p.M;
    a.K = p.K;
    a.n_slabs = p.n_slabs;
    a.nb = p.nb;
    a.B = b.B;
    a.TG = b.TG;
    a.frag = b.frag;
    a.tscale = b.tscale;
    a.step = b.step;
    const void* kern = b.TG == 1 ? (const void*)q4_batch_kernel<1> : (const void*)q4_batch_kernel<2>;
    cudaError_t e = ensure_smem_attr(kern, (int)BT_SMEM);
    if (e != cudaSuccess) return e;
    const uint32_t grid = std::min<uint32_t>(p.n_slabs, (uint32_t)device_sms());
    if (b.TG == 1) return launch_ex(q4_batch_kernel<1>, dim3(grid), dim3(BT_THREADS), BT_SMEM, st, true, a);
    return launch_ex(q4_batch_kernel<2>, dim3(grid), dim3(BT_THREADS), BT_SMEM, st, true, a);
}

// Tensor parallelism: in-place NCCL all-reduce of a batch buffer (the B
// partial residual updates of wo / down, B * dim floats; or the B argmax
// keys with max).  A no-op on one GPU.
static cudaError_t batch_allreduce(DevState* s, void* buf, size_t count, bool keys, cudaStream_t st) {
    if (s->tp_world == 1) return cudaSuccess;
    const NcclApi* n = nccl();
    if (!n || !s->comm) return cudaErrorUnknown;
    return nccl_status(keys ? n->all_reduce(buf, buf, count, ncclUint64, ncclMax, s->comm, st)
                            : n->all_reduce(buf, buf, count, ncclFloat32, ncclSum, s->comm, st));
}

static cudaError_t enqueue_batch_step(DevState* s, cudaStream_t st) {
    const BatchState& b = s->batch;
    const q_llama_config& c = s->cfg;
    const TpShape& t = s->tp;
    const uint32_t D = c.dim, H = t.h, L = c.n_layers;
    const size_t layer_floats = (size_t)t.nkv * c.max_seq_len * 2 * s->hd;
    cudaError_t e = cudaSuccess;
    auto prep = [&](const float* x, uint32_t ldx, uint32_t K, const float* norm, bool gather, float* copy) {
        BatchPrepArgs pa{};
        pa.x = x;
        pa.ldx = ldx;
        pa.gather = gather ? 1u : 0u;
        pa.step = b.step;
        pa.x_copy = copy;
        pa.norm_w = norm;
        pa.eps = c.rms_norm_eps;
        pa.K = K;
        pa.B = b.B;
        pa.TG = b.TG;
        pa.frag = b.frag;
        pa.tscale = b.tscale;
        return launch_xprep(s, pa, st);
    };
    for (uint32_t l = 0; l < L && e == cudaSuccess; ++l) {
        e = prep(l == 0 ? s->embd : b.x, D, D, s->attn_norm + (size_t)l * D, l == 0, l == 0 ? b.x : nullptr);
        if (e != cudaSuccess) break;
        BatchGemvArgs g{};
        g.epi = EPI_QKV;
        g.y = b.q;
        g.ldy = t.d;
        g.rope_cos = s->rope_cos;
        g.rope_sin = s->rope_sin;
        g.kv = b.d_pages ? b.kv : b.kv + (size_t)l * layer_floats;
        g.kv_seq_stride = (size_t)L * layer_floats;
        g.pages = b.d_pages;
        g.page_rows = b.page_rows;
        g.pages_per_seq = b.pages_per_seq;
        g.n_layers = L;
        g.layer = l;
        g.hd = s->hd;
        g.q_rows = t.d;
        g.kv_rows = t.kvd;
        g.max_seq = c.max_seq_len;
        if ((e = launch_bgemv(s, s->qkv[l], s->p_qkv, g, st)) != cudaSuccess) break;
        // attention: one cluster per (KV head, sequence)
        AttnArgs aa{};
        aa.q = b.q;
        aa.layer = l;
        aa.out = b.att;
        aa.step = b.step;
        aa.n_heads = t.nh;
        aa.n_kv_heads = t.nkv;
        aa.max_seq = c.max_seq_len;
        aa.chunk_alloc = b.att_ca;
        aa.slots = b.att_slots;
        aa.scale = 1.0f / sqrtf((float)s->hd);  // upstream model.c:1315
        aa.seq_stride = t.d;
        aa.n_layers = L;
        aa.pages = b.d_pages;
        aa.page_rows = b.page_rows;
        aa.pages_per_seq = b.pages_per_seq;
        {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(b.att_cs, t.nkv, b.B);
            cfg.blockDim = dim3(ATT_THREADS);
            cfg.dynamicSmemBytes = b.att_smem;
            cfg.stream = st;
            cudaLaunchAttribute attr[2];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = b.att_cs;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 2;
            const void* kern = attn_kernel_for(s->hd, c.n_heads / c.n_kv_heads);
            if (!kern) return cudaErrorInvalidValue;
            void* params[2] = {&aa, const_cast<CUtensorMap*>(&b.kv_map)};
            g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
            if ((e = cudaLaunchKernelExC(&cfg, kern, params)) != cudaSuccess) break;
        }
        if ((e = prep(b.att, t.d, t.d, nullptr, false, nullptr)) != cudaSuccess) break;
        g = BatchGemvArgs{};
        g.epi = residual_epi(s);  // tensor parallel: rank 0 adds the residual, the others their partial
        g.y = b.x;
        g.resid = b.x;
        g.ldy = D;
        if ((e = launch_bgemv(s, s->wo[l], s->p_wo, g, st)) != cudaSuccess) break;
        if ((e = batch_allreduce(s, b.x, (size_t)b.B * D, false, st)) != cudaSuccess) break;
        if ((e = prep(b.x, D, D, s->ffn_norm + (size_t)l * D, false, nullptr)) != cudaSuccess) break;
        g = BatchGemvArgs{};
        g.epi = EPI_SILU;
        g.y = b.h;
        g.ldy = H;
        if ((e = launch_bgemv(s, s->gu[l], s->p_gu, g, st)) != cudaSuccess) break;
        if ((e = prep(b.h, H, H, nullptr, false, nullptr)) != cudaSuccess) break;
        g = BatchGemvArgs{};
        g.epi = residual_epi(s);
        g.y = b.x;
        g.resid = b.x;
        g.ldy = D;
        if ((e = launch_bgemv(s, s->down[l], s->p_down, g, st)) != cudaSuccess) break;
        if ((e = batch_allreduce(s, b.x, (size_t)b.B * D, false, st)) != cudaSuccess) break;
    }
    if (e != cudaSuccess) return e;
    if ((e = prep(b.x, D, D, s->out_norm, false, nullptr)) != cudaSuccess) return e;
    BatchHeadArgs h{};
    h.w = s->out_w;
    h.V = t.v;
    h.row_base = t.v0;
    h.ldl = s->tp_world > 1 ? t.v_pad : t.v;
    h.K = D;
    h.B = b.B;
    h.TG = b.TG;
    h.wmul = b.wmul;
    h.wdiv = b.wdiv;
    h.frag = b.frag;
    h.tscale = b.tscale;
    h.logits = b.logits;
    h.best = b.best;
    const dim3 hg(2 * device_sms());
    e = b.TG == 1 ? launch_ex(batch_head_kernel<1>, hg, dim3(256), 0, st, true, h)
                  : launch_ex(batch_head_kernel<2>, hg, dim3(256), 0, st, true, h);
    if (e != cudaSuccess) return e;
    if ((e = batch_allreduce(s, b.best, b.B, true, st)) != cudaSuccess) return e;
    BatchAdvanceArgs ad{};
    ad.step = b.step;
    ad.best = b.best;
    ad.token_out = b.tok_out;
    ad.token_count = b.tok_count;
    ad.token_cap = b.tok_cap;
    ad.B = b.B;
    return launch_ex(batch_advance_kernel, dim3(1), dim3(32), 0, st, true, ad);
}

static constexpr uint32_t kNoPage = 0xFFFFFFFFu;

// page_rows == 0: contiguous caches (one upstream-layout cache per sequence);
// otherwise a pool of n_pages pages of page_rows rows (a multiple of the
// attention's 32-row stage) of every layer and KV head.
q_error_code batch_init(DevState* s, uint32_t B, uint32_t page_rows = 0, uint32_t n_pages = 0) {
    if (!s->built || (s->tp_world > 1 && !s->comm)) return Q_ERR_INVALID_ARG;
    if (B == 0 || B > BT_MAXB) return Q_ERR_INVALID_SIZE;
    const q_llama_config& c = s->cfg;
    const TpShape& t = s->tp;
    if ((size_t)std::max(c.dim, t.h) * 4 > 220 * 1024 || c.dim % 32 || t.h % 32) return Q_ERR_INVALID_CONFIG;
    Q_CUDA(cudaStreamSynchronize(s->stream));
    free_batch(s);
    BatchState& b = s->batch;
    b.B = B;
    b.TG = (B + 7) / 8;
    const size_t D = c.dim, V = c.vocab_size, Kmax = std::max<size_t>(D, t.h);
    b.tok_cap = c.max_seq_len;
    const size_t kv_seq = (size_t)c.n_layers * t.nkv * c.max_seq_len * 2 * s->hd * 4;
    b.kv_bytes_seq = kv_seq;
    const uint32_t sp = ATT_STAGE_BYTES / (s->hd * 4);  // attention stage rows
    if (page_rows) {
        if (page_rows % sp || page_rows > c.max_seq_len || n_pages == 0) {
            free_batch(s);
            return Q_ERR_INVALID_SIZE;
        }
        b.page_rows = page_rows;
        b.pages_per_seq = (c.max_seq_len + page_rows - 1) / page_rows;
        b.n_pages = n_pages;
    }
    const size_t kv_alloc = page_rows ? (size_t)n_pages * c.n_layers * t.nkv * page_rows * 2 * s->hd * 4 : kv_seq * B;
    if (!cuda_ok(dev_malloc(&b.kv, kv_alloc), "dev_malloc(batch kv)")) {
        free_batch(s);
        return Q_ERR_ALLOC_FAILED;
    }
    Q_CUDA(cudaMemset(b.kv, 0, kv_alloc));
    if (page_rows) {
        const size_t np = (size_t)B * b.pages_per_seq;
        if (!cuda_ok(dev_malloc(&b.d_pages, np * 4), "dev_malloc(page table)")) {
            free_batch(s);
            return Q_ERR_ALLOC_FAILED;
        }
        Q_CUDA(cudaMemset(b.d_pages, 0, np * 4));
        b.h_pages.assign(np, kNoPage);
        b.free_pages.resize(n_pages);
        for (uint32_t i = 0; i < n_pages; ++i) b.free_pages[i] = n_pages - 1 - i;  // pops 0, 1, 2, ...
    }
    if (s->tp_world > 1 &&
        !cuda_ok(dev_malloc(&b.gath, (size_t)s->tp_world * B * t.v_pad * 4), "dev_malloc(batch logits gather)")) {
        free_batch(s);
        return Q_ERR_ALLOC_FAILED;
    }
    {
        // the smallest cluster (2..16) that still gives every SM a CTA: at
        // 70B shapes and B = 16 that is 2 (measured per 70B layer: 345-381 us
        // at 2, 392 at 4, 401 at 8, 464 at 16, 368 at 1)
        uint32_t cs = 2;
        while (cs < 16 && (size_t)B * t.nkv * cs < (size_t)device_sms()) cs *= 2;
        const uint32_t G = c.n_heads / c.n_kv_heads;
        const uint32_t sp = ATT_STAGE_BYTES / (s->hd * 4);
        const uint32_t ca = ((c.max_seq_len + sp - 1) / sp + cs - 1) / cs * sp;
        const size_t limit = 227 * 1024 - 8 * 1024;
        b.att_slots = 0;
        for (uint32_t slots = ATT_MAX_SLOTS; slots >= 2 && !b.att_slots; --slots)
            if (attn_smem_bytes(G, s->hd, ca, slots) <= limit) {
                b.att_slots = slots;
                b.att_smem = attn_smem_bytes(G, s->hd, ca, slots);
            }
        if (!b.att_slots) {
            free_batch(s);
            return Q_ERR_INVALID_CONFIG;
        }
        b.att_cs = cs;
        b.att_ca = ca;
        const void* kern = attn_kernel_for(s->hd, G);
        if (cs > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        Q_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)std::max(b.att_smem, s->att_smem)));
    }
    const size_t sz[] = {bal(B * D * 4), bal(B * (size_t)t.d * 4), bal(B * (size_t)t.d * 4), bal(B * (size_t)t.h * 4),
                         bal(B * V * 4), bal(Kmax / 32 * b.TG * 32 * BT_FRAG_WORDS * 4), bal(BT_MAXB * 4),
                         bal(BT_MAXB * sizeof(StepParams)), bal(BT_MAXB * 8), bal((size_t)b.tok_cap * B * 4), bal(4),
                         bal(4)};
    size_t total = 0;
    for (size_t v : sz) total += v;
    if (!cuda_ok(dev_malloc(&b.base, total), "dev_malloc(batch state)")) {
        free_batch(s);
        return Q_ERR_ALLOC_FAILED;
    }
    uint8_t* p = b.base;
    b.x = (float*)p;
    p += sz[0];
    b.q = (float*)p;
    p += sz[1];
    b.att = (float*)p;
    p += sz[2];
    b.h = (float*)p;
    p += sz[3];
    b.logits = (float*)p;
    p += sz[4];
    b.frag = (uint32_t*)p;
    p += sz[5];
    b.tscale = (float*)p;
    p += sz[6];
    b.step = (StepParams*)p;
    p += sz[7];
    b.best = (unsigned long long*)p;
    p += sz[8];
    b.tok_out = (uint32_t*)p;
    p += sz[9];
    b.tok_count = (uint32_t*)p;
    p += sz[10];
    uint32_t* wmax = (uint32_t*)p;
    Q_CUDA(cudaMemset(b.base, 0, total));
    if (!cuda_ok(cudaMallocHost(&b.h_step, BT_MAXB * sizeof(StepParams)), "pinned batch steps")) {
        free_batch(s);
        return Q_ERR_ALLOC_FAILED;
    }
    // the LM head's power-of-two scale: max |W_out| into [2^14, 2^15)
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    absmax_kernel<<<2 * device_sms(), 256, 0, s->stream>>>(s->out_w, (size_t)t.v * D, wmax);
    uint32_t wm = 0;
    Q_CUDA(cudaMemcpyAsync(&wm, wmax, 4, cudaMemcpyDeviceToHost, s->stream));
    Q_CUDA(cudaStreamSynchronize(s->stream));
    int E = 0;
    const float mx = *reinterpret_cast<float*>(&wm);
    if (mx > 0.0f) frexpf(mx, &E);
    const int we = mx > 0.0f ? std::min(std::max(15 - E, -100), 100) : 0;
    b.wmul = ldexpf(1.0f, we);
    b.wdiv = ldexpf(1.0f, -we);
    // attention view of the B caches: planes (b * L + layer) * n_kv + head
    {
        const PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
        if (!encode) {
            free_batch(s);
            return Q_ERR_INVALID_ARG;
        }
        const uint32_t hd = s->hd;
        // contiguous: planes (b * L + layer) * n_kv + head of max_seq rows;
        // paged: planes (page * L + layer) * n_kv + head of page_rows rows
        const cuuint64_t rows = page_rows ? page_rows : c.max_seq_len;
        const cuuint64_t planes = (cuuint64_t)(page_rows ? n_pages : B) * c.n_layers * t.nkv;
        const cuuint64_t dims[3] = {2ull * hd, rows, planes};
        const cuuint64_t strides[2] = {2ull * hd * 4, 2ull * hd * 4 * rows};
        const cuuint32_t box[3] = {hd, ATT_STAGE_BYTES / (4 * hd), 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (encode(&b.kv_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, b.kv, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            set_last_error("cuTensorMapEncodeTiled(batch kv)", cudaErrorInvalidValue);
            free_batch(s);
            return Q_ERR_INVALID_ARG;
        }
    }
    // capture the step
    cudaStream_t st = s->stream;
    cudaGraph_t gr = nullptr;
    const uint64_t before = g_kernel_launches.load();
    if (!cuda_ok(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture")) {
        free_batch(s);
        return Q_ERR_INVALID_ARG;
    }
    cudaError_t e = enqueue_batch_step(s, st);
    const cudaError_t e2 = cudaStreamEndCapture(st, &gr);
    b.kernels = g_kernel_launches.load() - before;
    g_kernel_launches.fetch_sub(b.kernels);
    if (!cuda_ok(e, "batch capture") || !cuda_ok(e2, "batch end capture") ||
        !cuda_ok(cudaGraphInstantiate(&b.graph, gr, 0), "batch graph instantiate")) {
        if (gr) cudaGraphDestroy(gr);
        free_batch(s);
        return Q_ERR_INVALID_ARG;
    }
    cudaGraphDestroy(gr);
    return Q_OK;
}

// Paged caches: give sequence seq pages for its rows [0, rows) (zeroed when
// first given, as a contiguous cache starts zeroed).  Q_ERR_ARENA_OOM when
// the pool is exhausted.
static q_error_code batch_cover(DevState* s, uint32_t seq, uint64_t rows) {
    BatchState& b = s->batch;
    const uint64_t n = std::min<uint64_t>((rows + b.page_rows - 1) / b.page_rows, b.pages_per_seq);
    const size_t page_bytes = (size_t)s->cfg.n_layers * s->tp.nkv * b.page_rows * 2 * s->hd * 4;
    for (uint64_t r = 0; r < n; ++r) {
        uint32_t& e = b.h_pages[(size_t)seq * b.pages_per_seq + r];
        if (e != kNoPage) continue;
        if (b.free_pages.empty()) return Q_ERR_ARENA_OOM;
        e = b.free_pages.back();
        b.free_pages.pop_back();
        Q_CUDA(cudaMemsetAsync((uint8_t*)b.kv + (size_t)e * page_bytes, 0, page_bytes, s->stream));
        b.pages_dirty = true;
    }
    return Q_OK;
}

// The page table to the device before the next step reads it.
static q_error_code batch_sync_pages(DevState* s) {
    BatchState& b = s->batch;
    if (!b.d_pages || !b.pages_dirty) return Q_OK;
    Q_CUDA(cudaStreamSynchronize(s->stream));
    Q_CUDA(cudaMemcpy(b.d_pages, b.h_pages.data(), b.h_pages.size() * 4, cudaMemcpyHostToDevice));
    b.pages_dirty = false;
    return Q_OK;
}

}  // namespace qb200

using namespace qb200;

extern "C" {

q_error_code q_b200_batch_init_paged(q_context* ctx, q_llama_model* model, uint32_t batch, uint32_t page_rows,
                                     uint32_t n_pages) {
    if (!ctx || !model || page_rows == 0) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, false);
    if (!s) return Q_ERR_INVALID_ARG;
    return batch_init(s, batch, page_rows, n_pages);
}

q_error_code q_b200_batch_release(q_context* ctx, uint32_t seq) {
    if (!ctx) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, false);
    if (!s || !s->batch.kv || seq >= s->batch.B) return Q_ERR_INVALID_ARG;
    BatchState& b = s->batch;
    if (!b.d_pages) return Q_OK;  // contiguous caches: nothing to give back
    for (uint32_t r = 0; r < b.pages_per_seq; ++r) {
        uint32_t& e = b.h_pages[(size_t)seq * b.pages_per_seq + r];
        if (e == kNoPage) continue;
        b.free_pages.push_back(e);
        e = kNoPage;
        b.pages_dirty = true;
    }
    return Q_OK;
}

q_error_code q_b200_batch_init(q_context* ctx, q_llama_model* model, uint32_t batch) {
    if (!ctx || !model) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, false);
    if (!s) return Q_ERR_INVALID_ARG;
    return batch_init(s, batch);
}

static q_error_code batch_kv_io(q_context* ctx, uint32_t seq, size_t off, void* host, size_t bytes, bool write) {
    if (!ctx || !host) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, false);
    if (!s || !s->batch.kv) return Q_ERR_INVALID_ARG;
    if (seq >= s->batch.B) return Q_ERR_INVALID_ARG;
    const size_t n = s->batch.kv_bytes_seq;
    if (off > n || bytes > n - off) return Q_ERR_INVALID_SIZE;
    BatchState& b = s->batch;
    if (!b.d_pages) {
        uint8_t* d = (uint8_t*)b.kv + (size_t)seq * n + off;
        Q_CUDA(cudaStreamSynchronize(s->stream));
        Q_CUDA(write ? cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice)
                     : cudaMemcpy(host, d, bytes, cudaMemcpyDeviceToHost));
        return Q_OK;
    }
    // paged: whole rows of the upstream layout [L][n_kv][max_seq][K|V], copied
    // page by page; reading a row that has no page gives zeros
    const q_llama_config& c = s->cfg;
    const size_t rb = (size_t)2 * s->hd * 4, nkv = s->tp.nkv, ms = c.max_seq_len;
    if (off % rb || bytes % rb) return Q_ERR_INVALID_SIZE;
    const size_t page_bytes = (size_t)c.n_layers * nkv * b.page_rows * rb;
    for (size_t i = off / rb, end = (off + bytes) / rb; i < end;) {
        const size_t layer = i / (nkv * ms), head = (i / ms) % nkv, p = i % ms;
        const size_t r = p / b.page_rows, in = p % b.page_rows;
        const size_t run = std::min<size_t>({end - i, b.page_rows - in, ms - p});  // rows in this page and plane
        uint8_t* h = (uint8_t*)host + (i * rb - off);
        if (write) {
            q_error_code rc = batch_cover(s, seq, (uint64_t)(r + 1) * b.page_rows);
            if (rc != Q_OK) return rc;
        }
        const uint32_t pg = b.h_pages[(size_t)seq * b.pages_per_seq + r];
        if (pg == kNoPage) {
            std::memset(h, 0, run * rb);
        } else {
            uint8_t* d = (uint8_t*)b.kv + pg * page_bytes + ((layer * nkv + head) * b.page_rows + in) * rb;
            Q_CUDA(cudaStreamSynchronize(s->stream));
            Q_CUDA(write ? cudaMemcpy(d, h, run * rb, cudaMemcpyHostToDevice)
                         : cudaMemcpy(h, d, run * rb, cudaMemcpyDeviceToHost));
        }
        i += run;
    }
    return Q_OK;
}

q_error_code q_b200_batch_kv_write(q_context* ctx, uint32_t seq, size_t offset, const void* host, size_t bytes) {
    return batch_kv_io(ctx, seq, offset, const_cast<void*>(host), bytes, true);
}

q_error_code q_b200_batch_kv_read(q_context* ctx, uint32_t seq, size_t offset, void* host, size_t bytes) {
    return batch_kv_io(ctx, seq, offset, host, bytes, false);
}

q_error_code q_b200_decode_batch_loop(q_llama_model* model, q_context* ctx, const uint32_t* tokens,
                                      const uint32_t* pos, uint32_t n_steps, uint32_t* out_tokens, int sync) {
    if (!model || !ctx || !tokens || !pos) return Q_ERR_INVALID_ARG;
    if (n_steps == 0) return Q_ERR_INVALID_SIZE;
    DevState* s = state_of(ctx, false);
    if (!s || !s->built || !s->batch.graph) return Q_ERR_INVALID_ARG;
    BatchState& b = s->batch;
    const q_llama_config& c = model->config;
    for (uint32_t i = 0; i < b.B; ++i) {
        if (tokens[i] >= c.vocab_size) return Q_ERR_INVALID_ARG;
        if ((uint64_t)pos[i] + n_steps > c.max_seq_len) return Q_ERR_INVALID_ARG;
    }
    if (b.d_pages) {  // pages for every row the steps read or write
        for (uint32_t i = 0; i < b.B; ++i) {
            const q_error_code rc = batch_cover(s, i, (uint64_t)pos[i] + n_steps);
            if (rc != Q_OK) return rc;
        }
        const q_error_code rc = batch_sync_pages(s);
        if (rc != Q_OK) return rc;
    }
    Q_CUDA(cudaStreamSynchronize(s->stream));  // h_step may still be read by a prior copy
    for (uint32_t i = 0; i < b.B; ++i) {
        b.h_step[i].token = tokens[i];
        b.h_step[i].pos = pos[i];
        b.h_step[i].n_row = b.h_step[i].valid = pos[i] + 1;
    }
    Q_CUDA(cudaMemcpyAsync(b.step, b.h_step, b.B * sizeof(StepParams), cudaMemcpyHostToDevice, s->stream));
    Q_CUDA(cudaMemsetAsync(b.tok_count, 0, 4, s->stream));
    for (uint32_t i = 0; i < n_steps; ++i) {
        Q_CUDA(cudaGraphLaunch(b.graph, s->stream));
        g_kernel_launches.fetch_add(b.kernels);
    }
    if (!sync) return Q_OK;
    Q_CUDA(cudaStreamSynchronize(s->stream));
    q_error_code rc = check_device_status("q_b200_decode_batch_loop");
    if (rc != Q_OK) return rc;
    if (out_tokens) {
        const uint32_t n = std::min(n_steps, b.tok_cap);
        Q_CUDA(cudaMemcpy(out_tokens, b.tok_out, (size_t)n * b.B * 4, cudaMemcpyDeviceToHost));
    }
    return Q_OK;
}

q_error_code q_b200_decode_batch(q_llama_model* model, q_context* ctx, const uint32_t* tokens, const uint32_t* pos,
                                 float* logits, uint32_t* next_tokens) {
    q_error_code rc = q_b200_decode_batch_loop(model, ctx, tokens, pos, 1, next_tokens, 1);
    if (rc != Q_OK) return rc;
    DevState* s = state_of(ctx, false);
    if (!logits) return Q_OK;
    const BatchState& b = s->batch;
    const uint32_t V = model->config.vocab_size;
    if (s->tp_world == 1) {
        Q_CUDA(cudaMemcpy(logits, b.logits, (size_t)b.B * V * 4, cudaMemcpyDeviceToHost));
        return Q_OK;
    }
    // every rank's [B][v_pad] rows, gathered in rank order (a collective: all
    // ranks call this together, as they do llama_forward), then reordered
    const NcclApi* n = nccl();
    if (!n || !s->comm) return Q_ERR_INVALID_ARG;
    const size_t per = (size_t)b.B * s->tp.v_pad;
    Q_CUDA(nccl_status(n->all_gather(b.logits, b.gath, per, ncclFloat32, s->comm, s->stream)));
    std::vector<float> all(per * s->tp_world);
    Q_CUDA(cudaMemcpyAsync(all.data(), b.gath, all.size() * 4, cudaMemcpyDeviceToHost, s->stream));
    Q_CUDA(cudaStreamSynchronize(s->stream));
    for (uint32_t r = 0; r < s->tp_world; ++r) {
        const uint32_t v0 = std::min(V, r * s->tp.v_pad), v1 = std::min(V, v0 + s->tp.v_pad);
        for (uint32_t q = 0; q < b.B; ++q)
            std::memcpy(logits + (size_t)q * V + v0, all.data() + r * per + (size_t)q * s->tp.v_pad,
                        (size_t)(v1 - v0) * 4);
    }
    return Q_OK;
}

}  // extern "C"
