// prefill.cu — host side of the prompt path (kernels in prefill.cuh).
//
// A prompt of S > 1 rows at positions pos..pos+S-1 runs layer by layer as
// dense contractions instead of upstream's row-by-row GEMVs
// (src/models/model.c:1120-1165):
//
//   per layer: X = RMSNorm(x) -> halves; W_qkv -> halves; Y = X W^T with the
//   RoPE + KV-store epilogue; causal attention over the cache; O -> halves;
//   x += O W_o^T; X = RMSNorm(x) -> halves; x_h = SiLU(X W_g^T) * (X W_u^T);
//   x += x_h W_down^T
//
// then the LM head on the last row only (upstream model.c:1799-1844) and the
// step advance, so a decode step can follow at once.  The workspace (~1 GB
// at the 8B shape and 2048 rows) is allocated on the first prompt and kept;
// decode steps never touch it.
#include "runtime.cuh"

namespace qb200 {

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

static q_error_code prefill_workspace(DevState* s, uint32_t S) {
    if (S <= s->pf_cap) return Q_OK;
    const q_llama_config& c = s->cfg;
    const TpShape& t = s->tp;
    const uint32_t cap = (S + 127) / 128 * 128;
    const size_t D = c.dim, Kmax = std::max<size_t>(D, t.h);
    const size_t Mmax = std::max<size_t>(std::max<size_t>(t.d + 2 * t.kvd, 2 * t.h), D);
    const size_t sz_tok = al256((size_t)cap * 4), sz_x = al256((size_t)cap * D * 4);
    const size_t sz_act = al256((size_t)2 * cap * Kmax * 2), sz_ts = al256((size_t)cap * 4);
    const size_t sz_q = al256((size_t)cap * t.d * 4), sz_h = al256((size_t)cap * t.h * 4);
    const size_t sz_w = al256(2 * Mmax * Kmax * 2), sz_rs = al256(Mmax * 4);
    const size_t total = sz_tok + sz_x + sz_act + sz_ts + 2 * sz_q + sz_h + sz_w + sz_rs;
    Q_CUDA(cudaStreamSynchronize(s->stream));
    if (s->pf_base) cudaFree(s->pf_base);
    if (s->pf_tok_host) cudaFreeHost(s->pf_tok_host);
    s->pf_base = nullptr;
    s->pf_tok_host = nullptr;
    s->pf_cap = 0;
    if (!cuda_ok(dev_malloc(&s->pf_base, total), "dev_malloc(prefill workspace)")) return Q_ERR_ALLOC_FAILED;
    if (!cuda_ok(cudaMallocHost(&s->pf_tok_host, (size_t)cap * 4), "pinned prompt ids")) return Q_ERR_ALLOC_FAILED;
    uint8_t* p = s->pf_base;
    s->pf_tok = (uint32_t*)p;
    p += sz_tok;
    s->pf_x = (float*)p;
    p += sz_x;
    s->pf_act = (__half*)p;
    p += sz_act;
    s->pf_tscale = (float*)p;
    p += sz_ts;
    s->pf_q = (float*)p;
    p += sz_q;
    s->pf_o = (float*)p;
    p += sz_q;
    s->pf_h = (float*)p;
    p += sz_h;
    s->pf_w = (__half*)p;
    p += sz_w;
    s->pf_rscale = (float*)p;
    s->pf_cap = cap;
    return Q_OK;
}

// 3-D map over [2 (hi, lo)][rows][K] fp16 halves: boxes of PF_BK x box_rows,
// 128-byte swizzle (the layout the MMA descriptors expect).
static bool halves_map(CUtensorMap* m, const __half* base, uint32_t rows, uint32_t K, uint32_t box_rows) {
    const PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[3] = {K, rows, 2};
    const cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)rows * K * 2};
    const cuuint32_t box[3] = {PF_BK, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_last_error("cuTensorMapEncodeTiled(prefill operand)", cudaErrorInvalidValue);
        return false;
    }
    return true;
}

static cudaError_t launch_act_split(DevState* s, const ActSplitArgs& a, uint32_t S, cudaStream_t st) {
    const size_t smem = (size_t)a.K * 4;
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    // one attribute per kernel and device: the opt-in maximum covers every K
    cudaError_t e = ensure_smem_attr((const void*)act_split_kernel, 227 * 1024);
    if (e != cudaSuccess) return e;
    (void)s;
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    act_split_kernel<<<S, 256, smem, st>>>(a);
    return cudaGetLastError();
}

static cudaError_t launch_w_split(DevState* s, const uint8_t* packed, const GemvPlan& p, cudaStream_t st) {
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    w_split_kernel<<<p.n_slabs, 256, 0, st>>>(packed, p.M, p.nb, s->pf_w, s->pf_w + (size_t)p.M * p.K,
                                               s->pf_rscale);
    return cudaGetLastError();
}

// Y = X W^T for X = the activation halves [S][K], W = the weight halves [M][K].
static cudaError_t launch_pf_gemm(DevState* s, uint32_t S, uint32_t M, uint32_t K, PfGemmArgs a, cudaStream_t st) {
    CUtensorMap ma, mb;
    if (!halves_map(&ma, s->pf_act, S, K, PF_BM) || !halves_map(&mb, s->pf_w, M, K, PF_BN))
        return cudaErrorInvalidValue;
    a.S = S;
    a.M = M;
    a.K = K;
    a.n_mt = (S + PF_BM - 1) / PF_BM;
    a.n_nt = (M + PF_BN - 1) / PF_BN;
    a.tscale = s->pf_tscale;
    a.rscale = s->pf_rscale;
    cudaError_t e = ensure_smem_attr((const void*)pf_gemm_kernel, (int)PF_SMEM);
    if (e != cudaSuccess) return e;
    const uint32_t tiles = a.n_mt * a.n_nt;
    const uint32_t grid = std::min<uint32_t>(tiles, (uint32_t)device_sms());
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    pf_gemm_kernel<<<grid, PF_THREADS, PF_SMEM, st>>>(ma, mb, a);
    return cudaGetLastError();
}

static const void* pf_attn_tc_kernel_g(uint32_t G) {
    switch (G) {
        case 1: return (const void*)attn_prefill_tc_kernel<128, 1>;
        case 2: return (const void*)attn_prefill_tc_kernel<128, 2>;
        case 4: return (const void*)attn_prefill_tc_kernel<128, 4>;
        case 8: return (const void*)attn_prefill_tc_kernel<128, 8>;
        default: return nullptr;
    }
}

template <int HD>
static const void* pf_attn_kernel_g(uint32_t G) {
    switch (G) {
        case 1: return (const void*)attn_prefill_kernel<HD, 1>;
        case 2: return (const void*)attn_prefill_kernel<HD, 2>;
        case 4: return (const void*)attn_prefill_kernel<HD, 4>;
        case 8: return (const void*)attn_prefill_kernel<HD, 8>;
        default: return nullptr;
    }
}

static cudaError_t launch_pf_attention(DevState* s, float* kv, uint32_t layer, uint32_t S, uint32_t pos,
                                       cudaStream_t st) {
    const q_llama_config& c = s->cfg;
    const uint32_t G = c.n_heads / c.n_kv_heads, hd = s->hd;
    // head_dim 128 (the Llama-3 shapes): tensor cores; smaller heads: CUDA cores
    const bool tc = hd == 128;
    const void* kern = tc ? pf_attn_tc_kernel_g(G)
                          : hd == 32 ? pf_attn_kernel_g<32>(G) : hd == 64 ? pf_attn_kernel_g<64>(G) : nullptr;
    if (!kern) return cudaErrorInvalidValue;
    const size_t smem = tc ? pf_attn_tc_smem(hd) : pf_attn_smem(hd);
    cudaError_t e = ensure_smem_attr(kern, (int)smem);
    if (e != cudaSuccess) return e;
    PfAttnArgs a{};
    a.q = s->pf_q;
    a.kv = kv + (size_t)layer * s->tp.nkv * c.max_seq_len * 2 * hd;
    a.out = s->pf_o;
    a.S = S;
    a.pos = pos;
    a.n_heads = s->tp.nh;
    a.n_kv = s->tp.nkv;
    a.max_seq = c.max_seq_len;
    a.scale = 1.0f / sqrtf((float)hd);  // upstream model.c:1315
    const uint32_t rq = (tc ? PT_Q : PF_ATT_Q) / G;
    dim3 grid((S + rq - 1) / rq, s->tp.nkv);
    void* params[1] = {&a};
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernel(kern, grid, dim3(tc ? PT_THREADS : PF_ATT_THREADS), params, smem, st);
}

// Tensor parallelism: in-place sum of the S x dim partial residuals over the
// ranks (NCCL; 32 MB at 2048 rows of the 8B shape).  A no-op on one GPU.
static cudaError_t pf_allreduce(DevState* s, float* buf, size_t count, cudaStream_t st) {
    if (s->tp_world == 1) return cudaSuccess;
    const NcclApi* n = nccl();
    if (!n || !s->comm) return cudaErrorUnknown;
    return nccl_status(n->all_reduce(buf, buf, count, ncclFloat32, ncclSum, s->comm, st));
}

q_error_code run_prefill(DevState* s, float* kv, const uint32_t* tokens, uint32_t S, uint32_t pos, bool sample) {
    const q_llama_config& c = s->cfg;
    const TpShape& t = s->tp;
    if (s->tp_world != 1 && !s->comm) return Q_ERR_INVALID_ARG;
    q_error_code rc = prefill_workspace(s, S);
    if (rc != Q_OK) return rc;
    cudaStream_t st = s->stream;
    const uint32_t D = c.dim, H = t.h;
    std::memcpy(s->pf_tok_host, tokens, (size_t)S * 4);
    Q_CUDA(cudaMemcpyAsync(s->pf_tok, s->pf_tok_host, (size_t)S * 4, cudaMemcpyHostToDevice, st));
    const size_t layer_floats = (size_t)t.nkv * c.max_seq_len * 2 * s->hd;
    __half* hi = s->pf_act;
    auto lo_of = [&](uint32_t K) { return s->pf_act + (size_t)S * K; };
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        // attention block
        ActSplitArgs as{};
        as.x = l == 0 ? s->embd : s->pf_x;
        as.tokens = l == 0 ? s->pf_tok : nullptr;
        as.ldx = D;
        as.x_copy = l == 0 ? s->pf_x : nullptr;
        as.norm_w = s->attn_norm + (size_t)l * D;
        as.eps = c.rms_norm_eps;
        as.K = D;
        as.hi = hi;
        as.lo = lo_of(D);
        as.tscale = s->pf_tscale;
        Q_CUDA(launch_act_split(s, as, S, st));
        Q_CUDA(launch_w_split(s, s->qkv[l], s->p_qkv, st));
        PfGemmArgs g{};
        g.epi = EPI_QKV;
        g.y = s->pf_q;
        g.ldy = t.d;
        g.rope_cos = s->rope_cos;
        g.rope_sin = s->rope_sin;
        g.kv_layer = kv + (size_t)l * layer_floats;
        g.hd = s->hd;
        g.q_rows = t.d;
        g.kv_rows = t.kvd;
        g.max_seq = c.max_seq_len;
        g.pos = pos;
        Q_CUDA(launch_pf_gemm(s, S, s->p_qkv.M, D, g, st));
        Q_CUDA(launch_pf_attention(s, kv, l, S, pos, st));
        as = ActSplitArgs{};
        as.x = s->pf_o;
        as.ldx = t.d;
        as.K = t.d;
        as.hi = hi;
        as.lo = lo_of(t.d);
        as.tscale = s->pf_tscale;
        Q_CUDA(launch_act_split(s, as, S, st));
        Q_CUDA(launch_w_split(s, s->wo[l], s->p_wo, st));
        g = PfGemmArgs{};
        g.epi = residual_epi(s);  // tensor parallel: rank 0 adds the residual, the others their partial
        g.y = s->pf_x;
        g.resid = s->pf_x;
        g.ldy = D;
        Q_CUDA(launch_pf_gemm(s, S, D, t.d, g, st));
        Q_CUDA(pf_allreduce(s, s->pf_x, (size_t)S * D, st));
        // feed-forward block
        as = ActSplitArgs{};
        as.x = s->pf_x;
        as.ldx = D;
        as.norm_w = s->ffn_norm + (size_t)l * D;
        as.eps = c.rms_norm_eps;
        as.K = D;
        as.hi = hi;
        as.lo = lo_of(D);
        as.tscale = s->pf_tscale;
        Q_CUDA(launch_act_split(s, as, S, st));
        Q_CUDA(launch_w_split(s, s->gu[l], s->p_gu, st));
        g = PfGemmArgs{};
        g.epi = EPI_SILU;
        g.y = s->pf_h;
        g.ldy = H;
        Q_CUDA(launch_pf_gemm(s, S, 2 * H, D, g, st));
        as = ActSplitArgs{};
        as.x = s->pf_h;
        as.ldx = H;
        as.K = H;
        as.hi = hi;
        as.lo = lo_of(H);
        as.tscale = s->pf_tscale;
        Q_CUDA(launch_act_split(s, as, S, st));
        Q_CUDA(launch_w_split(s, s->down[l], s->p_down, st));
        g = PfGemmArgs{};
        g.epi = residual_epi(s);
        g.y = s->pf_x;
        g.resid = s->pf_x;
        g.ldy = D;
        Q_CUDA(launch_pf_gemm(s, S, D, H, g, st));
        Q_CUDA(pf_allreduce(s, s->pf_x, (size_t)S * D, st));
    }
    // last row: LM head + argmax, then the step advance (the next decode
    // step then runs at pos + S with the argmax as its token)
    StepParams* hp = &s->h_step[0];
    hp->token = tokens[S - 1];
    hp->pos = pos + S - 1;
    hp->n_row = pos + S;
    hp->valid = pos + S;
    Q_CUDA(cudaMemcpyAsync(s->step, hp, sizeof *hp, cudaMemcpyHostToDevice, st));
    Q_CUDA(enqueue_head(s, st, s->pf_x + (size_t)(S - 1) * D, sample));
    return Q_OK;
}

}  // namespace qb200
