// runtime.cu — launch plans, error plumbing and the per-context device-state
// registry of libqorus_b200.so.
#include <cmath>
#include <cstdio>

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
    static std::once_flag once;
    static cudaStream_t s = nullptr;
    std::call_once(once, [] { cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking); });
    return s;
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

bool plan_gemv(uint32_t M, uint32_t K, bool pairs, GemvPlan& p) {
    if (M == 0 || K == 0 || K % 32) return false;
    const uint32_t nb = K / 32;
    uint32_t R = 1;
    while (R * 2 <= 128 && (uint64_t)R * 2 * nb * 20 <= 24576) R *= 2;
    if (pairs && R < 2) R = 2;
    while ((R * nb) % 4) R *= 2;  // tiles are whole 16-byte units
    uint32_t bpt = 0, c = 0;
    for (uint32_t b = 1; b <= 2 && !bpt; b *= 2) {
        if (nb % b) continue;
        const uint32_t nbc = nb / b;
        for (uint32_t cc = R; cc >= 1; cc /= 2) {
            const uint32_t T = nbc * cc;
            if (T <= (uint32_t)GEMV_MAX_CONSUMERS && T % 32 == 0) {
                bpt = b;
                c = cc;
                break;
            }
        }
    }
    if (!bpt) return false;
    if (R / c > 4) R = 4 * c;  // kernels are instantiated for 1, 2 or 4 rows per thread
    if ((R * nb) % 4) return false;
    p.M = M;
    p.K = K;
    p.R = R;
    p.c = c;
    p.bpt = bpt;
    p.n_tiles = (M + R - 1) / R;
    p.grid = std::min<uint32_t>(p.n_tiles, 2u * (uint32_t)device_sms());  // 2 CTAs per SM
    p.threads = nb / bpt * c + 32;
    p.smem = gemv_smem_bytes(R, K, bpt);
    p.packed_bytes = (size_t)p.n_tiles * gemv_tile_bytes(R, K);
    return true;
}

cudaError_t launch_gemv(const GemvPlan& p, GemvArgs a, cudaStream_t s, bool pdl) {
    a.M = p.M;
    a.K = p.K;
    a.R = p.R;
    a.c = p.c;
    a.bpt = p.bpt;
    a.n_tiles = p.n_tiles;
    using Kern = void (*)(GemvArgs);
    static const Kern table[2][3] = {
        {gemv_q4_kernel<1, 1>, gemv_q4_kernel<1, 2>, gemv_q4_kernel<1, 4>},
        {gemv_q4_kernel<2, 1>, gemv_q4_kernel<2, 2>, gemv_q4_kernel<2, 4>}};
    static std::once_flag once;
    std::call_once(once, [] {
        for (auto& row : table)
            for (Kern k : row)
                cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    const uint32_t rows = p.R / p.c;
    const int ri = rows == 1 ? 0 : rows == 2 ? 1 : rows == 4 ? 2 : -1;
    if (ri < 0 || (p.bpt != 1 && p.bpt != 2)) return cudaErrorInvalidValue;
    return launch_ex(table[p.bpt - 1][ri], dim3(p.grid), dim3(p.threads), p.smem, s, pdl, a);
}

cudaError_t pack_q4(const uint8_t* d_aos, const GemvPlan& p, uint32_t interleave_half,
                    uint8_t* d_dst, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(d_dst, 0, p.packed_bytes, s);
    if (e != cudaSuccess) return e;
    const uint64_t n = (uint64_t)p.M * (p.K / 32);
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 65535);
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    q4_pack_kernel<<<blocks, 256, 0, s>>>(d_aos, p.M, p.K, p.R, interleave_half, d_dst);
    return cudaGetLastError();
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
    s->g_body = s->g_full = nullptr;
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
