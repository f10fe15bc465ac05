// api_ops.cu — upstream kernel-level entry points (host buffers in and out,
// computed on the GPU) and their device-pointer counterparts.
//
// Validation mirrors the upstream functions (src/ops/avx2/*.c): null
// pointers -> Q_ERR_INVALID_ARG, 32-byte alignment -> Q_ERR_MISALIGNED,
// sizes -> Q_ERR_INVALID_SIZE, aliasing -> Q_ERR_ALIASING, dtype ->
// Q_ERR_INVALID_DTYPE.  Each call copies its operands to the device, runs
// the kernel on the library's op stream and copies the result back; these
// are convenience paths, not the model hot path.
#include <cstdlib>

#include "runtime.cuh"

using namespace qb200;

namespace {

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    bool alloc(size_t n) { return cuda_ok(dev_malloc(&p, n ? n : 16), "dev_malloc(op)"); }
    float* f() { return (float*)p; }
};

bool aligned32(const void* p) { return ((uintptr_t)p & 31) == 0; }

q_error_code to_dev(DevBuf& b, const void* h, size_t n) {
    if (!b.alloc(n)) return Q_ERR_ALLOC_FAILED;
    if (!cuda_ok(cudaMemcpyAsync(b.p, h, n, cudaMemcpyHostToDevice, op_stream()), "op h2d"))
        return Q_ERR_INVALID_ARG;
    return Q_OK;
}

q_error_code finish(void* host_out, const void* dev, size_t n) {
    if (!cuda_ok(cudaGetLastError(), "op launch")) return Q_ERR_INVALID_ARG;
    if (!cuda_ok(cudaMemcpyAsync(host_out, dev, n, cudaMemcpyDeviceToHost, op_stream()), "op d2h"))
        return Q_ERR_INVALID_ARG;
    if (!cuda_ok(cudaStreamSynchronize(op_stream()), "op sync")) return Q_ERR_INVALID_ARG;
    return check_device_status("op");
}

}  // namespace

extern "C" {

// ---- Q4_0 GEMV -------------------------------------------------------------------

size_t q_b200_q4_packed_bytes(uint32_t M, uint32_t K) {
    GemvPlan p;
    return plan_gemv(M, K, p) ? p.packed_bytes : 0;
}

q_error_code q_b200_q4_pack(const q_block_q4_0* d_src, uint32_t M, uint32_t K, void* d_dst,
                            void* stream) {
    if (!d_src || !d_dst) return Q_ERR_INVALID_ARG;
    GemvPlan p;
    if (!plan_gemv(M, K, p)) return Q_ERR_INVALID_SIZE;
    Q_CUDA(pack_q4((const uint8_t*)d_src, p, 0, (uint8_t*)d_dst, (cudaStream_t)stream));
    return Q_OK;
}

q_error_code q_b200_gemv_q4(const void* d_packed, uint32_t M, uint32_t K, const float* d_x,
                            float* d_y, void* stream) {
    if (!d_packed || !d_x || !d_y) return Q_ERR_INVALID_ARG;
    if (d_x == d_y) return Q_ERR_ALIASING;
    if (((uintptr_t)d_x & 15) || ((uintptr_t)d_packed & 15)) return Q_ERR_MISALIGNED;
    GemvPlan p;
    ChainPlan cp;
    if (!plan_single(M, K, p, cp)) return Q_ERR_INVALID_SIZE;
    GemvArgs a{};
    a.w = (const uint8_t*)d_packed;
    a.x = d_x;
    a.y = d_y;
    a.epi = EPI_STORE;
    void* scratch = op_gemv_scratch(cp.scratch_bytes());
    if (!scratch) return Q_ERR_ALLOC_FAILED;
    Q_CUDA(launch_single(cp, p, a, scratch, (cudaStream_t)stream));
    return Q_OK;
}

// upstream matmul.c:98-271 validation, then pack + GEMV on the device
q_error_code q_gemv_q4_f32_avx2(const q_tensor* w, const float* x, float* y) {
    if (!w || !x || !y) return Q_ERR_INVALID_ARG;
    if (!aligned32(x) || !aligned32(y)) return Q_ERR_MISALIGNED;
    if (x == y) return Q_ERR_ALIASING;
    const uint32_t M = w->ne[0], K = w->ne[1];
    if (M == 0 || K == 0 || K % 32) return Q_ERR_INVALID_SIZE;
    if (w->type != Q_Q4_0) return Q_ERR_INVALID_DTYPE;
    const uint32_t nb = K / 32;
    if (nb > UINT32_MAX / M) return Q_ERR_OVERFLOW;
    if (w->nb[0] != (size_t)nb * sizeof(q_block_q4_0)) return Q_ERR_INVALID_ARG;
    if (!w->data) return Q_ERR_INVALID_ARG;
    GemvPlan p;
    ChainPlan cp;
    if (!plan_single(M, K, p, cp)) return Q_ERR_INVALID_SIZE;
    DevBuf aos, packed, dx, dy;
    q_error_code rc;
    if ((rc = to_dev(aos, w->data, (size_t)M * nb * 20)) || (rc = to_dev(dx, x, (size_t)K * 4)))
        return rc;
    if (!packed.alloc(p.packed_bytes) || !dy.alloc((size_t)M * 4)) return Q_ERR_ALLOC_FAILED;
    Q_CUDA(pack_q4((const uint8_t*)aos.p, p, 0, (uint8_t*)packed.p, op_stream()));
    GemvArgs a{};
    a.w = (const uint8_t*)packed.p;
    a.x = dx.f();
    a.y = dy.f();
    a.epi = EPI_STORE;
    void* scratch = op_gemv_scratch(cp.scratch_bytes());
    if (!scratch) return Q_ERR_ALLOC_FAILED;
    Q_CUDA(launch_single(cp, p, a, scratch, op_stream()));
    return finish(y, dy.p, (size_t)M * 4);
}

q_error_code q_b200_gemv_f32(const float* d_w, uint32_t M, uint32_t K, const float* d_x,
                             float* d_y, void* stream) {
    if (!d_w || !d_x || !d_y) return Q_ERR_INVALID_ARG;
    if (M == 0 || K == 0 || K % 4) return Q_ERR_INVALID_SIZE;
    if (((uintptr_t)d_w & 15) || ((uintptr_t)d_x & 15)) return Q_ERR_MISALIGNED;
    HeadArgs h{};
    h.slots = head_slots(K);
    if (!h.slots) return Q_ERR_INVALID_SIZE;
    h.w = d_w;
    h.x = d_x;
    h.rows = M;
    h.K = K;
    h.logits = d_y;
    Q_CUDA(ensure_smem_attr((const void*)lm_head_kernel, 227 * 1024));
    const uint32_t grid = std::max<uint32_t>(1, std::min<uint32_t>(device_sms(), M));
    Q_CUDA(launch_ex(lm_head_kernel, dim3(grid), dim3(HEAD_THREADS), head_smem_bytes(K, h.slots),
                     (cudaStream_t)stream, false, h));
    return Q_OK;
}

// ---- elementwise / normalisation --------------------------------------------------

q_error_code q_rmsnorm_f32_avx2(const float* x, const float* w, float* out, uint32_t N, float eps) {
    if (!x || !w || !out) return Q_ERR_INVALID_ARG;
    if (!aligned32(x) || !aligned32(w) || !aligned32(out)) return Q_ERR_MISALIGNED;
    if (N == 0 || N % 8) return Q_ERR_INVALID_SIZE;
    DevBuf dx, dw, d;
    q_error_code rc;
    if ((rc = to_dev(dx, x, (size_t)N * 4)) || (rc = to_dev(dw, w, (size_t)N * 4))) return rc;
    if (!d.alloc((size_t)N * 4)) return Q_ERR_ALLOC_FAILED;
    g_kernel_launches++;
    rmsnorm_kernel<<<1, OPS_THREADS, 0, op_stream()>>>(dx.f(), dw.f(), d.f(), N, eps);
    return finish(out, d.p, (size_t)N * 4);
}

q_error_code q_rope_f32_avx2(const float* x, const float* c, const float* s, float* out, uint32_t N) {
    if (!x || !c || !s || !out) return Q_ERR_INVALID_ARG;
    if (!aligned32(x) || !aligned32(c) || !aligned32(s) || !aligned32(out)) return Q_ERR_MISALIGNED;
    if (N == 0 || N % 8) return Q_ERR_INVALID_SIZE;
    DevBuf dx, dc, ds, d;
    q_error_code rc;
    if ((rc = to_dev(dx, x, (size_t)N * 4)) || (rc = to_dev(dc, c, (size_t)N * 4)) ||
        (rc = to_dev(ds, s, (size_t)N * 4)))
        return rc;
    if (!d.alloc((size_t)N * 4)) return Q_ERR_ALLOC_FAILED;
    g_kernel_launches++;
    rope_kernel<<<(N / 2 + 255) / 256, 256, 0, op_stream()>>>(dx.f(), dc.f(), ds.f(), d.f(), N);
    return finish(out, d.p, (size_t)N * 4);
}

q_error_code q_silu_f32_avx2(const float* x, float* out, uint32_t N) {
    if (!x || !out) return Q_ERR_INVALID_ARG;
    if (N == 0) return Q_ERR_INVALID_SIZE;
    if (N >= 8 && (!aligned32(x) || !aligned32(out))) return Q_ERR_MISALIGNED;
    DevBuf dx, d;
    q_error_code rc;
    if ((rc = to_dev(dx, x, (size_t)N * 4))) return rc;
    if (!d.alloc((size_t)N * 4)) return Q_ERR_ALLOC_FAILED;
    g_kernel_launches++;
    silu_kernel<<<std::min<uint32_t>((N + 255) / 256, 4096), 256, 0, op_stream()>>>(dx.f(), d.f(), N);
    return finish(out, d.p, (size_t)N * 4);
}

q_error_code q_softmax_f32_avx2(const float* x, float* out, uint32_t N) {
    if (!x || !out) return Q_ERR_INVALID_ARG;
    if (N == 0) return Q_ERR_INVALID_SIZE;
    if (N >= 8 && (!aligned32(x) || !aligned32(out))) return Q_ERR_MISALIGNED;
    DevBuf dx, d;
    q_error_code rc;
    if ((rc = to_dev(dx, x, (size_t)N * 4))) return rc;
    if (!d.alloc((size_t)N * 4)) return Q_ERR_ALLOC_FAILED;
    g_kernel_launches++;
    softmax_kernel<<<1, OPS_THREADS, 0, op_stream()>>>(dx.f(), d.f(), N);
    return finish(out, d.p, (size_t)N * 4);
}

static q_error_code binary(const q_tensor* a, const q_tensor* b, q_tensor* o, int op) {
    if (!a || !b || !o || !a->data || !b->data || !o->data) return Q_ERR_INVALID_ARG;
    for (const q_tensor* t : {a, b, (const q_tensor*)o})
        if (t->ne[1] != 1 || t->ne[2] != 1 || t->ne[3] != 1) return Q_ERR_INVALID_SIZE;
    const uint32_t N = a->ne[0];
    if (N != b->ne[0] || N != o->ne[0]) return Q_ERR_INVALID_SIZE;
    if (a->type != Q_F32 || b->type != Q_F32 || o->type != Q_F32) return Q_ERR_INVALID_DTYPE;
    if (N == 0) return Q_ERR_INVALID_SIZE;
    DevBuf da, db, d;
    q_error_code rc;
    if ((rc = to_dev(da, a->data, (size_t)N * 4)) || (rc = to_dev(db, b->data, (size_t)N * 4)))
        return rc;
    if (!d.alloc((size_t)N * 4)) return Q_ERR_ALLOC_FAILED;
    g_kernel_launches++;
    binary_kernel<<<std::min<uint32_t>((N + 255) / 256, 4096), 256, 0, op_stream()>>>(
        da.f(), db.f(), d.f(), N, op);
    return finish(o->data, d.p, (size_t)N * 4);
}

q_error_code q_add_f32_avx2(const q_tensor* a, const q_tensor* b, q_tensor* o) { return binary(a, b, o, 0); }
q_error_code q_mul_f32_avx2(const q_tensor* a, const q_tensor* b, q_tensor* o) { return binary(a, b, o, 1); }

q_error_code q_causal_mask_f32_avx2(q_tensor* s, float mask) {
    if (!s || !s->data) return Q_ERR_INVALID_ARG;
    if (s->type != Q_F32) return Q_ERR_INVALID_DTYPE;
    const uint32_t n = s->ne[0];
    if (n == 0 || s->ne[1] != n) return Q_ERR_INVALID_SIZE;
    const size_t ld = s->nb[0] / 4;
    if (ld < n) return Q_ERR_INVALID_SIZE;
    const size_t bytes = ((size_t)(n - 1) * ld + n) * 4;
    DevBuf d;
    q_error_code rc;
    if ((rc = to_dev(d, s->data, bytes))) return rc;
    g_kernel_launches++;
    causal_mask_kernel<<<256, 256, 0, op_stream()>>>(d.f(), n, ld, mask);
    return finish(s->data, d.p, bytes);
}

// C = A B; B in upstream's two forms (matmul_fp32.c:195-289): a transposed
// view (nb[0] == 4, columns K apart) or row-major with stride nb[0]/4.
q_error_code q_matmul_f32_avx2(const q_tensor* A, const q_tensor* B, q_tensor* C, q_context* ctx) {
    if (!A || !B || !C || !ctx) return Q_ERR_INVALID_ARG;
    const uint32_t M = A->ne[0], K = A->ne[1], N = B->ne[1];
    if (M == 0 || K == 0 || N == 0) return Q_ERR_INVALID_SIZE;
    if (B->ne[0] != K || C->ne[0] != M || C->ne[1] != N) return Q_ERR_INVALID_SIZE;
    if (A->type != Q_F32 || B->type != Q_F32 || C->type != Q_F32) return Q_ERR_INVALID_DTYPE;
    if (!A->data || !B->data || !C->data) return Q_ERR_INVALID_ARG;
    const size_t sa = A->nb[0] / 4, sb = B->nb[0] / 4, sc = C->nb[0] / 4;
    if (sa < K || sc < N) return Q_ERR_INVALID_SIZE;
    const bool tr = B->nb[0] == 4 && B->ne[0] > 1 && B->nb[1] > 4;
    if (tr && B->nb[1] / 4 < K) return Q_ERR_INVALID_SIZE;
    if (!tr && sb < N) return Q_ERR_INVALID_SIZE;
    const size_t a_bytes = ((size_t)(M - 1) * sa + K) * 4;
    const size_t b_bytes = tr ? (size_t)N * K * 4 : ((size_t)(K - 1) * sb + N) * 4;
    const size_t c_bytes = ((size_t)(M - 1) * sc + N) * 4;
    DevBuf da, db, dc;
    q_error_code rc;
    if ((rc = to_dev(da, A->data, a_bytes)) || (rc = to_dev(db, B->data, b_bytes)) ||
        (rc = to_dev(dc, C->data, c_bytes)))
        return rc;
    g_kernel_launches++;
    const uint64_t n = (uint64_t)M * N;
    matmul_f32_kernel<<<(uint32_t)std::min<uint64_t>((n + 255) / 256, 8192), 256, 0, op_stream()>>>(
        da.f(), sa, 1, db.f(), tr ? 1 : sb, tr ? K : 1, dc.f(), sc, M, N, K);
    return finish(C->data, dc.p, c_bytes);
}

void q_dequantize_q4_0_block_avx2_public(const q_block_q4_0* block, float* output) {
    if (!block || !output) return;
    DevBuf db, d;
    if (to_dev(db, block, sizeof(q_block_q4_0)) || !d.alloc(32 * 4)) return;
    g_kernel_launches++;
    dequant_block_kernel<<<1, 32, 0, op_stream()>>>((const uint8_t*)db.p, d.f());
    finish(output, d.p, 32 * 4);
}

}  // extern "C"

// ---- Q4_0 GEMM over many rows (the prefill contraction) ------------------------------

namespace {
struct GemmWork {
    void* p = nullptr;
    size_t bytes = 0;
};
}  // namespace

extern "C" q_error_code q_b200_gemm_q4(const void* d_packed, uint32_t M, uint32_t K, const float* d_x,
                                       uint32_t n_rows, float* d_y, void* stream) {
    if (!d_packed || !d_x || !d_y) return Q_ERR_INVALID_ARG;
    if (n_rows == 0) return Q_ERR_INVALID_SIZE;
    if ((const void*)d_x == (const void*)d_y) return Q_ERR_ALIASING;
    if (((uintptr_t)d_x & 15) || ((uintptr_t)d_packed & 15) || ((uintptr_t)d_y & 15)) return Q_ERR_MISALIGNED;
    GemvPlan p;
    if (!plan_gemv(M, K, p)) return Q_ERR_INVALID_SIZE;
    // workspace: activation halves [2][n][K], weight halves [2][M][K], scales
    static std::mutex mu;
    static std::unordered_map<int, GemmWork> work;
    std::lock_guard<std::mutex> lk(mu);
    int dev = 0;
    Q_CUDA(cudaGetDevice(&dev));
    const size_t b_act = ((size_t)2 * n_rows * K * 2 + 255) / 256 * 256;
    const size_t b_w = ((size_t)2 * M * K * 2 + 255) / 256 * 256;
    const size_t b_ts = ((size_t)n_rows * 4 + 255) / 256 * 256, b_rs = ((size_t)M * 4 + 255) / 256 * 256;
    const size_t need = b_act + b_w + b_ts + b_rs;
    GemmWork& w = work[dev];
    cudaStream_t st = (cudaStream_t)stream;
    if (w.bytes < need) {
        Q_CUDA(cudaDeviceSynchronize());
        if (w.p) cudaFree(w.p);
        w = GemmWork{};
        if (!cuda_ok(dev_malloc(&w.p, need), "dev_malloc(gemm workspace)")) return Q_ERR_ALLOC_FAILED;
        w.bytes = need;
    }
    uint8_t* base = (uint8_t*)w.p;
    DevState tmp;  // only the prefill workspace fields are used
    tmp.pf_act = (__half*)base;
    tmp.pf_w = (__half*)(base + b_act);
    tmp.pf_tscale = (float*)(base + b_act + b_w);
    tmp.pf_rscale = (float*)(base + b_act + b_w + b_ts);
    ActSplitArgs as{};
    as.x = d_x;
    as.ldx = K;
    as.K = K;
    as.hi = tmp.pf_act;
    as.lo = tmp.pf_act + (size_t)n_rows * K;
    as.tscale = tmp.pf_tscale;
    Q_CUDA(launch_act_split(&tmp, as, n_rows, st));
    Q_CUDA(launch_w_split(&tmp, (const uint8_t*)d_packed, p, st));
    PfGemmArgs g{};
    g.epi = EPI_STORE;
    g.y = d_y;
    g.ldy = M;
    Q_CUDA(launch_pf_gemm(&tmp, n_rows, M, K, g, st));
    return Q_OK;
}

// ---- device status and bounded waits ---------------------------------------------

extern "C" {

q_error_code q_b200_set_wait_limit_ns(uint64_t ns) {
    if (ns == 0) return Q_ERR_INVALID_ARG;
    const unsigned long long v = ns;
    Q_CUDA(cudaMemcpyToSymbol(g_qdev_wait_ns, &v, sizeof v));
    return Q_OK;
}

uint32_t q_b200_device_status(void) { return take_device_status(); }

q_error_code q_b200_selftest_exchange_timeout(uint64_t limit_ns, uint32_t* status_out) {
    if (!status_out || limit_ns == 0) return Q_ERR_INVALID_ARG;
    *status_out = 0;
    // A single-rank receive of the fused tensor-parallel exchange whose
    // sender never runs: every CTA's wait for the tagged words must give up
    // after limit_ns.
    GemvPlan p;
    ChainPlan cp;
    if (!plan_single(64, 256, p, cp)) return Q_ERR_INVALID_SIZE;
    const uint32_t slice = 256;
    const size_t xb = tp_buffer_bytes(1, slice);
    DevBuf w, y, ex;
    if (!w.alloc(p.packed_bytes) || !y.alloc(64 * 4) || !ex.alloc(xb)) return Q_ERR_ALLOC_FAILED;
    void* scratch = op_gemv_scratch(cp.scratch_bytes());
    if (!scratch) return Q_ERR_ALLOC_FAILED;
    cudaStream_t st = op_stream();
    Q_CUDA(cudaMemsetAsync(w.p, 0, p.packed_bytes, st));
    Q_CUDA(cudaMemsetAsync(ex.p, 0, xb, st));
    Q_CUDA(cudaStreamSynchronize(st));
    if (take_device_status() != 0) return Q_ERR_INVALID_ARG;  // an earlier error is not ours
    unsigned long long old = 0;
    Q_CUDA(cudaMemcpyFromSymbol(&old, g_qdev_wait_ns, sizeof old));
    const unsigned long long lim = limit_ns;
    Q_CUDA(cudaMemcpyToSymbol(g_qdev_wait_ns, &lim, sizeof lim));
    GemvArgs a{};
    a.w = (const uint8_t*)w.p;
    a.x = y.f();  // unused: the input comes from the receive slots
    a.y = y.f();
    a.epi = EPI_STORE;
    GemvTp t{};
    t.tp_base[0] = (uint8_t*)ex.p;
    t.tp_off = (uint32_t)tp_fused_offset(1, slice);
    t.tp_slice = slice;
    t.tp_world = 1;
    t.tp_rank = 0;
    t.tp_recv = 1;
    t.tp_par = 0;
    const GemvPlan* m[1] = {&p};
    const cudaError_t e = launch_chain(cp, m, &a, scratch, nullptr, nullptr, st, false, &t);
    const cudaError_t e2 = cudaStreamSynchronize(st);
    cudaMemcpyToSymbol(g_qdev_wait_ns, &old, sizeof old);
    Q_CUDA(e);
    Q_CUDA(e2);
    *status_out = take_device_status();
    return Q_OK;
}

}  // extern "C"
