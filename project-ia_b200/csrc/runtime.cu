// runtime.cu — launch plans, error plumbing and the per-context device-state
// registry of libqorus_b200.so.
#include <cmath>
#include <cstdio>
#include <set>

#include "runtime.cuh"

namespace qb200 {

std::atomic<uint64_t> g_kernel_launches{0};
static std::mutex g_err_mu;
static std::string g_last_error;

void set_last_error(const char* where, cudaError_t e) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
}

const char* last_error_cstr() {
    std::lock_guard<std::mutex> lk(g_err_mu);
    return g_last_error.c_str();
}

bool cuda_ok(cudaError_t e, const char* where) {
    if (e == cudaSuccess) return true;
    set_last_error(where, e);
    return false;
}

int device_sms() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

cudaStream_t op_stream() {
    static std::mutex mu;
    static std::unordered_map<int, cudaStream_t> streams;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    cudaStream_t& s = streams[dev];
    if (!s) cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    return s;
}

cudaError_t ensure_smem_attr(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({kernel, dev})) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({kernel, dev});
    return e;
}

q_error_code check_device_status(const char* where) {
    uint32_t st = 0;
    if (!cuda_ok(cudaMemcpyFromSymbol(&st, g_qdev_status, sizeof st), where)) return Q_ERR_INVALID_ARG;
    if (st != 0) {
        {
            std::lock_guard<std::mutex> lk(g_err_mu);
            g_last_error = std::string(where) + ": device wait timed out (code " + std::to_string(st) + ")";
        }
        uint32_t zero = 0;
        cudaMemcpyToSymbol(g_qdev_status, &zero, sizeof zero);
        return Q_ERR_INVALID_ARG;
    }
    return Q_OK;
}

// ---- GEMV plans -----------------------------------------------------------------
// R: largest power of two with a ~24 KB tile (4-stage ring ~96 KB, so the
// next kernel's CTA fits beside this one under programmatic dependent
// launch).  Threads: (nb/bpt)*c <= 256, a multiple of 32.

bool plan_gemv(uint32_t M, uint32_t K, GemvPlan& p) {
    if (M == 0 || K == 0 || K % 32) return false;
    const uint32_t nb = K / 32, n_slabs = (M + 15) / 16;
    if (n_slabs > GemvPlan::kTicketWords) return false;
    const uint64_t NB = (uint64_t)n_slabs * nb;
    const int sms = device_sms();
#ifndef QB200_GEMV_STAGE_BLOCKS
#define QB200_GEMV_STAGE_BLOCKS 64  // 20 KB stages
#endif
    uint32_t stage_blocks = QB200_GEMV_STAGE_BLOCKS;
#ifndef QB200_GEMV_PER_SM
#define QB200_GEMV_PER_SM 2
#endif
#ifndef QB200_GEMV_MAX_STAGES
#define QB200_GEMV_MAX_STAGES 8
#endif
    uint32_t per_sm = QB200_GEMV_PER_SM, n_stage = 0;
    // two CTAs per SM (the next kernel's CTA also fits under programmatic
    // dependent launch) when a >= 2-stage ring fits in ~113 KB, else one
    uint32_t red_slabs = 1;
    for (; per_sm >= 1; --per_sm) {
        // slabs one CTA's range touches (at most), held in shared memory
        // between CTA-wide reductions (capped: longer ranges reduce in batches)
        const uint64_t grid = std::min<uint64_t>(NB, (uint64_t)per_sm * sms);
        const uint64_t range = (NB + grid - 1) / grid;
        red_slabs = (uint32_t)std::min<uint64_t>(32, (range + nb - 1) / nb + 1);
        const size_t fixed = gemv_smem_bytes(nb, 0, 0, red_slabs);
        const size_t budget = per_sm == 2 ? 113 * 1024 : 220 * 1024;
        if (budget <= fixed) continue;
        n_stage = (uint32_t)std::min<size_t>(QB200_GEMV_MAX_STAGES,
                                             (budget - fixed) / (stage_blocks * GEMV_BLOCK_BYTES));
        if (n_stage >= 2) break;
    }
    if (per_sm < 1 || n_stage < 2) return false;
    p.M = M;
    p.K = K;
    p.n_slabs = n_slabs;
    p.nb = nb;
    p.stage_blocks = stage_blocks;
    p.n_stage = n_stage;
    p.grid = (uint32_t)std::min<uint64_t>(NB, (uint64_t)per_sm * sms);
    if (NB * p.grid >= (1ull << 32)) return false;  // the kernel's range math is 32-bit
    const uint64_t per_cta = std::max<uint64_t>(1, NB / p.grid);
    p.max_parts = (uint32_t)((nb + per_cta - 1) / per_cta + 2);
    p.red_slabs = red_slabs;
    p.smem = gemv_smem_bytes(nb, stage_blocks, n_stage, red_slabs);
    p.packed_bytes = (size_t)NB * GEMV_BLOCK_BYTES;
    return true;
}

cudaError_t launch_gemv(const GemvPlan& p, GemvArgs a, void* scratch, cudaStream_t s, bool pdl) {
    a.M = p.M;
    a.K = p.K;
    a.n_slabs = p.n_slabs;
    a.nb = p.nb;
    a.stage_blocks = p.stage_blocks;
    a.n_stage = p.n_stage;
    a.max_parts = p.max_parts;
    a.red_slabs = p.red_slabs;
    a.ticket = reinterpret_cast<uint32_t*>(scratch);
    a.part = reinterpret_cast<float*>(a.ticket + GemvPlan::kTicketWords);
    const cudaError_t e = ensure_smem_attr((const void*)gemv_q4_kernel, 220 * 1024);
    if (e != cudaSuccess) return e;
    return launch_ex(gemv_q4_kernel, dim3(p.grid), dim3(GEMV_THREADS), p.smem, s, pdl, a);
}

cudaError_t pack_q4(const uint8_t* d_aos, const GemvPlan& p, uint32_t interleave_half,
                    uint8_t* d_dst, cudaStream_t s) {
    const uint64_t n = (uint64_t)p.n_slabs * p.nb * 32;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 65535);
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    q4_pack_kernel<<<blocks, 256, 0, s>>>(d_aos, p.M, p.K, interleave_half, d_dst);
    return cudaGetLastError();
}

void* op_gemv_scratch(const GemvPlan& p) {
    static std::mutex mu;
    static std::unordered_map<int, std::pair<void*, size_t>> bufs;  // device -> buffer
    std::lock_guard<std::mutex> lk(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    auto& b = bufs[dev];
    if (b.second < p.scratch_bytes()) {
        if (b.first) {
            cudaDeviceSynchronize();
            cudaFree(b.first);
        }
        b = {nullptr, 0};
        void* q = nullptr;
        if (!cuda_ok(cudaMalloc(&q, p.scratch_bytes()), "cudaMalloc(gemv scratch)")) return nullptr;
        if (!cuda_ok(cudaMemset(q, 0, p.scratch_bytes()), "memset(gemv scratch)")) return nullptr;
        b = {q, p.scratch_bytes()};
    }
    return b.first;
}

// ---- per-context registry ---------------------------------------------------------

static std::mutex g_reg_mu;
static std::unordered_map<const q_context*, DevState*> g_reg;

DevState* state_of(const q_context* ctx, bool create) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    auto it = g_reg.find(ctx);
    if (it != g_reg.end()) return it->second;
    if (!create) return nullptr;
    DevState* s = new DevState();
    cudaGetDevice(&s->device);
    if (!cuda_ok(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "stream")) {
        delete s;
        return nullptr;
    }
    g_reg[ctx] = s;
    return s;
}

void state_erase(const q_context* ctx) {
    DevState* s = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_reg_mu);
        auto it = g_reg.find(ctx);
        if (it == g_reg.end()) return;
        s = it->second;
        g_reg.erase(it);
    }
    cudaStreamSynchronize(s->stream);
    free_model(s);
    if (s->arena) cudaFree(s->arena);
    if (s->h_step) cudaFreeHost(s->h_step);
    cudaStreamDestroy(s->stream);
    delete s;
}

void* dev_arena_alloc(DevState* s, size_t bytes) {
    const size_t a = Q_ALIGN_SIZE(bytes ? bytes : 1);
    if (!s->arena || s->arena_head + a > s->arena_size) return nullptr;
    void* p = s->arena + s->arena_head;
    s->arena_head += a;
    return p;
}

void free_model(DevState* s) {
    if (s->g_body) cudaGraphExecDestroy(s->g_body);
    if (s->g_full) cudaGraphExecDestroy(s->g_full);
    if (s->g_trace) cudaGraphExecDestroy(s->g_trace);
    if (s->trace_buf) cudaFree(s->trace_buf);
    s->trace_buf = nullptr;
    s->g_body = s->g_full = s->g_trace = nullptr;
    s->graph_kv = nullptr;
    for (void* p : s->weight_allocs) cudaFree(p);
    s->weight_allocs.clear();
    s->qkv.clear();
    s->wo.clear();
    s->gu.clear();
    s->down.clear();
    s->built = false;
}

}  // namespace qb200
