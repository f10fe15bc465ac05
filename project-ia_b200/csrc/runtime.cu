// runtime.cu — launch plans, error plumbing and the per-context device-state
// registry of libqorus_b200.so.
#include <cmath>
#include <cstdio>
#include <set>
#include <tuple>

#include "runtime.cuh"

namespace qb200 {

std::atomic<uint64_t> g_kernel_launches{0};
std::atomic<uint64_t> g_device_allocs{0};
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
    // the opt-in limit covers static + dynamic shared memory
    cudaFuncAttributes fa{};
    int optin = 0;
    if ((e = cudaFuncGetAttributes(&fa, kernel)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
        return e;
    bytes = std::min(bytes, optin - (int)fa.sharedSizeBytes);
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({kernel, dev});
    return e;
}

// ---- areas kernels leave zero between launches --------------------------------

static std::mutex g_zero_mu;
static std::vector<std::tuple<int, void*, size_t>> g_zero_areas;  // (device, ptr, bytes)

void register_zero_area(void* p, size_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_zero_mu);
    g_zero_areas.emplace_back(dev, p, bytes);
}

void unregister_zero_area(void* p) {
    std::lock_guard<std::mutex> lk(g_zero_mu);
    g_zero_areas.erase(std::remove_if(g_zero_areas.begin(), g_zero_areas.end(),
                                      [p](const auto& t) { return std::get<1>(t) == p; }),
                       g_zero_areas.end());
}

uint32_t take_device_status() {
    uint32_t st = 0;
    if (cudaMemcpyFromSymbol(&st, g_qdev_status, sizeof st) != cudaSuccess) return QDEV_BAD_ARG;
    if (st == 0) return 0;
    // A wait that gave up may have left tickets or barrier counters
    // non-zero; the next launch needs them zero.  Everything in flight on
    // the device finishes first.
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceSynchronize();
    {
        std::lock_guard<std::mutex> lk(g_zero_mu);
        for (const auto& t : g_zero_areas)
            if (std::get<0>(t) == dev) cudaMemset(std::get<1>(t), 0, std::get<2>(t));
    }
    const uint32_t zero = 0;
    cudaMemcpyToSymbol(g_qdev_status, &zero, sizeof zero);
    cudaDeviceSynchronize();
    return st;
}

q_error_code check_device_status(const char* where) {
    const uint32_t st = take_device_status();
    if (st != 0) {
        std::lock_guard<std::mutex> lk(g_err_mu);
        g_last_error = std::string(where) + ": device wait timed out (code " + std::to_string(st) + ")";
        return Q_ERR_INVALID_ARG;
    }
    return Q_OK;
}

// ---- GEMV plans -----------------------------------------------------------------

bool plan_gemv(uint32_t M, uint32_t K, GemvPlan& p) {
    if (M == 0 || K == 0 || K % 32) return false;
    const uint32_t nb = K / 32, n_slabs = (M + GEMV_SLAB_ROWS - 1) / GEMV_SLAB_ROWS;
    if (n_slabs > ChainPlan::kTicketWords) return false;
    p.M = M;
    p.K = K;
    p.n_slabs = n_slabs;
    p.nb = nb;
    p.packed_bytes = (size_t)p.NB() * GEMV_BLOCK_BYTES;
    return true;
}

// Grid: one CTA per SM (GEMV_CONSUMER_WARPS consumer warps each), fewer when a
// phase has fewer tiles.  Every CTA takes an equal contiguous share of each
// phase's tile stream.  Ring: the largest stage (256, 192, 128, 64 tiles)
// that leaves room for >= 2 stages beside the input tables; as many stages
// as fit.
bool plan_chain(const GemvPlan* const* mats, uint32_t n, ChainPlan& cp) {
    if (n == 0 || n > (uint32_t)GEMV_MAX_PHASES) return false;
    constexpr uint32_t kMaxStages = 8;      // ring depth cap
    constexpr uint32_t kWholeSlabPct = 60;  // smallest whole-slab grid, % of the SMs
    uint64_t grid = device_sms();  // one CTA per SM
    uint32_t max_nb = 0;
    for (uint32_t i = 0; i < n; ++i) {
        grid = std::min<uint64_t>(grid, mats[i]->NB());
        max_nb = std::max(max_nb, mats[i]->nb);
    }
    if (grid == 0) return false;
    // Whole slabs: a grid that divides the slab count gives every CTA the
    // same whole slabs, so no slab is split across CTAs and no partial sums
    // or tickets are needed.  Worth it while the grid still covers most
    // SMs (measured: 96 of 148 SMs still stream these matrices at close to the
    // full HBM rate, and the split-slab finish costs more than the idle SMs).
    if (n == 1) {
        const uint64_t ns = mats[0]->n_slabs;
        for (uint64_t d = std::min<uint64_t>(grid, ns); d >= 1; --d) {
            if (ns % d) continue;
            if (d * 100 >= (uint64_t)device_sms() * kWholeSlabPct) grid = d;
            break;
        }
    }
    cp = ChainPlan{};
    cp.n = n;
    cp.grid = (uint32_t)grid;
    cp.max_nb = max_nb;
    uint32_t red_slabs = 1;
    for (uint32_t i = 0; i < n; ++i) {
        const GemvPlan& m = *mats[i];
        const uint64_t NB = m.NB();
        if (NB * grid >= (1ull << 32)) return false;  // the kernel's range math is 32-bit
        const uint64_t per_cta = std::max<uint64_t>(1, NB / grid);
        cp.max_parts[i] = (uint32_t)((m.nb + per_cta - 1) / per_cta + 2);
        cp.part_floats = std::max<size_t>(cp.part_floats, (size_t)m.n_slabs * cp.max_parts[i] * GEMV_SLAB_ROWS);
        // slabs one CTA's range touches, held in shared memory between
        // CTA-wide reductions (capped: longer ranges reduce in batches)
        const uint64_t range = (NB + grid - 1) / grid;
        red_slabs = std::max<uint32_t>(red_slabs, (uint32_t)std::min<uint64_t>(8, (range + m.nb - 1) / m.nb + 1));
    }
    cp.red_slabs = red_slabs;
    const size_t budget = 220 * 1024;
    const size_t fixed = gemv_smem_bytes(max_nb, 0, 0, red_slabs);
    if (fixed >= budget) return false;
    const uint32_t sizes[] = {256, 192, 128, 64, 32, 16};  // the small ones for K up to ~28K
    for (uint32_t sb : sizes) {
        const uint32_t ns = (uint32_t)std::min<size_t>(kMaxStages,
                                                       (budget - fixed) / ((size_t)sb * GEMV_BLOCK_BYTES));
        if (ns >= 2) {
            cp.stage_blocks = sb;
            cp.n_stage = ns;
            break;
        }
    }
    if (cp.n_stage < 2) return false;
    cp.smem = gemv_smem_bytes(max_nb, cp.stage_blocks, cp.n_stage, red_slabs);
    return true;
}

cudaError_t launch_chain(const ChainPlan& cp, const GemvPlan* const* mats, const GemvArgs* args,
                         void* scratch, uint32_t* bar, unsigned long long* trace, cudaStream_t s,
                         bool pdl, const GemvTp* tp) {
    GemvChain c{};
    for (uint32_t i = 0; i < cp.n; ++i) {
        GemvArgs a = args[i];
        a.M = mats[i]->M;
        a.K = mats[i]->K;
        a.n_slabs = mats[i]->n_slabs;
        a.nb = mats[i]->nb;
        a.max_parts = cp.max_parts[i];
        a.ticket = reinterpret_cast<uint32_t*>(scratch);
        a.part = reinterpret_cast<float*>(a.ticket + ChainPlan::kTicketWords);
        c.ph[i] = a;
    }
    c.n_phases = cp.n;
    c.stage_blocks = cp.stage_blocks;
    c.n_stage = cp.n_stage;
    c.red_slabs = cp.red_slabs;
    c.max_nb = cp.max_nb;
    c.bar = bar;
    c.trace = trace;
    if (cp.n > 1 && !bar) return cudaErrorInvalidValue;
    const bool fused = tp && (tp->tp_send || tp->tp_recv);
    if (fused && cp.n != 1) return cudaErrorInvalidValue;
    if (fused) c.tp = *tp;
    const void* kern = fused ? (const void*)q4_slab_kernel<true> : (const void*)q4_slab_kernel<false>;
    cudaError_t e = ensure_smem_attr(kern, 227 * 1024);
    if (e != cudaSuccess) return e;
    // Phases after the first wait on the whole grid: all CTAs must be
    // resident at once (cooperative launch).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cp.grid);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = cp.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    uint32_t na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cp.n > 1) {
        attr[na].id = cudaLaunchAttributeCooperative;
        attr[na].val.cooperative = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    void* params[1] = {&c};
    return cudaLaunchKernelExC(&cfg, kern, params);
}

bool plan_single(uint32_t M, uint32_t K, GemvPlan& p, ChainPlan& cp) {
    if (!plan_gemv(M, K, p)) return false;
    const GemvPlan* m[1] = {&p};
    return plan_chain(m, 1, cp);
}

cudaError_t launch_single(const ChainPlan& cp, const GemvPlan& p, const GemvArgs& a, void* scratch,
                          cudaStream_t s) {
    const GemvPlan* m[1] = {&p};
    // programmatic dependent launch: back-to-back GEMVs on one stream stream
    // the next one's weights during this one's tail (the kernel waits for the
    // previous grid before it reads its input or touches its scratch)
    return launch_chain(cp, m, &a, scratch, nullptr, nullptr, s, true);
}

cudaError_t pack_q4(const uint8_t* d_aos, const GemvPlan& p, uint32_t interleave_half,
                    uint8_t* d_dst, cudaStream_t s) {
    const uint64_t n = (uint64_t)p.n_slabs * p.nb * 32;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 65535);
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    q4_pack_kernel<<<blocks, 256, 0, s>>>(d_aos, p.M, p.K, interleave_half, d_dst);
    return cudaGetLastError();
}

void* op_gemv_scratch(size_t bytes) {
    static std::mutex mu;
    static std::unordered_map<int, std::pair<void*, size_t>> bufs;  // device -> buffer
    std::lock_guard<std::mutex> lk(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    auto& b = bufs[dev];
    if (b.second < bytes) {
        if (b.first) {
            cudaDeviceSynchronize();
            unregister_zero_area(b.first);
            cudaFree(b.first);
        }
        b = {nullptr, 0};
        void* q = nullptr;
        if (!cuda_ok(dev_malloc(&q, bytes), "dev_malloc(gemv scratch)")) return nullptr;
        if (!cuda_ok(cudaMemset(q, 0, bytes), "memset(gemv scratch)")) return nullptr;
        b = {q, bytes};
        register_zero_area(q, ChainPlan::kTicketWords * 4);
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
    if (s->comm) {
        if (const NcclApi* n = nccl()) n->comm_destroy(s->comm);
        s->comm = nullptr;
    }
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
    free_batch(s);
    if (s->g_body) cudaGraphExecDestroy(s->g_body);
    if (s->g_full) cudaGraphExecDestroy(s->g_full);
    if (s->g_trace) cudaGraphExecDestroy(s->g_trace);
    if (s->g_sample) cudaGraphExecDestroy(s->g_sample);
    s->g_sample = nullptr;
    if (s->trace_buf) cudaFree(s->trace_buf);
    s->trace_buf = nullptr;
    s->g_body = s->g_full = s->g_trace = nullptr;
    s->graph_kv = nullptr;
    if (s->gemv_scratch) unregister_zero_area(s->gemv_scratch);
    if (s->chain_bar) unregister_zero_area(s->chain_bar);
    s->gemv_scratch = nullptr;
    s->chain_bar = nullptr;
    for (void* p : s->weight_allocs) cudaFree(p);
    s->weight_allocs.clear();
    if (s->pf_base) cudaFree(s->pf_base);
    if (s->pf_tok_host) cudaFreeHost(s->pf_tok_host);
    if (s->samp_probs) cudaFree(s->samp_probs);
    s->samp_probs = nullptr;
    s->samp_keep = nullptr;
    s->pf_base = nullptr;
    s->pf_tok_host = nullptr;
    s->pf_cap = 0;
    s->qkv.clear();
    s->wo.clear();
    s->gu.clear();
    s->down.clear();
    s->built = false;
}

}  // namespace qb200
