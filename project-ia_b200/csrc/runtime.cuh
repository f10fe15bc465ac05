// runtime.cuh — host-side state shared by the parts of libqorus_b200.so:
// launch plans, per-context device state, error plumbing.
#pragma once

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <cudaTypedefs.h>

#include "attn_decode.cuh"
#include "gemv_q4.cuh"
#include "head.cuh"
#include "ops.cuh"
#include "prefill.cuh"
#include "sample.cuh"
#include "batch.cuh"
#include "qorus_b200.h"
#include "tp.cuh"

namespace qb200 {

// ---- errors / counters ------------------------------------------------------

void set_last_error(const char* where, cudaError_t e);
bool cuda_ok(cudaError_t e, const char* where);
const char* last_error_cstr();
extern std::atomic<uint64_t> g_kernel_launches;
extern std::atomic<uint64_t> g_device_allocs;
// cudaMalloc, counted (q_b200_device_allocations): every device allocation of
// the library goes through here.
inline cudaError_t dev_malloc(void** p, size_t bytes) {
    g_device_allocs.fetch_add(1, std::memory_order_relaxed);
    return cudaMalloc(p, bytes);
}
template <typename T>
inline cudaError_t dev_malloc(T** p, size_t bytes) {
    return dev_malloc(reinterpret_cast<void**>(p), bytes);
}
int device_sms();
cudaStream_t op_stream();  // stream for the kernel-level entry points (per device)
// cudaFuncAttributeMaxDynamicSharedMemorySize = bytes for `kernel` on the
// current device (set once per kernel and device).
cudaError_t ensure_smem_attr(const void* kernel, int bytes);

#define Q_CUDA(call)                                                    \
    do {                                                                \
        if (!::qb200::cuda_ok((call), #call)) return Q_ERR_INVALID_ARG; \
    } while (0)

// ---- GEMV launch plans -----------------------------------------------------------

// One matrix: shape, slab tiling, packed size.
struct GemvPlan {
    uint32_t M = 0, K = 0, n_slabs = 0, nb = 0;
    size_t packed_bytes = 0;
    uint64_t NB() const { return (uint64_t)n_slabs * nb; }
};

// A chain of 1..GEMV_MAX_PHASES matrices run by one persistent grid (one
// CTA per SM).  Scratch layout, shared by every plan: a fixed ticket area of
// kTicketWords uint32 (zero between launches: each finisher resets its
// ticket), then the partial sums [n_slabs][max_parts][32] fp32 of the
// largest phase.
struct ChainPlan {
    uint32_t n = 0, grid = 0, stage_blocks = 0, n_stage = 0, red_slabs = 0, max_nb = 0;
    uint32_t max_parts[GEMV_MAX_PHASES] = {};
    size_t smem = 0, part_floats = 0;
    static constexpr size_t kTicketWords = 16384;
    size_t scratch_bytes() const { return kTicketWords * 4 + part_floats * 4; }
};

bool plan_gemv(uint32_t M, uint32_t K, GemvPlan& p);
bool plan_chain(const GemvPlan* const* mats, uint32_t n, ChainPlan& cp);
// args[i]: phase i's pointers and epilogue; shapes, tiling and scratch
// pointers are filled in here.  scratch: cp.scratch_bytes() whose ticket
// words are zero before the first launch (kernels leave them zero); bar:
// cp.n zeroed counters when cp.n > 1 (likewise left zero).
cudaError_t launch_chain(const ChainPlan& cp, const GemvPlan* const* mats, const GemvArgs* args,
                         void* scratch, uint32_t* bar, unsigned long long* trace, cudaStream_t s,
                         bool pdl, const GemvTp* tp = nullptr);
// One GEMV on its own (a one-phase chain).
bool plan_single(uint32_t M, uint32_t K, GemvPlan& p, ChainPlan& cp);
cudaError_t launch_single(const ChainPlan& cp, const GemvPlan& p, const GemvArgs& a, void* scratch,
                          cudaStream_t s);
cudaError_t pack_q4(const uint8_t* d_aos, const GemvPlan& p, uint32_t interleave_half,
                    uint8_t* d_dst, cudaStream_t s);
// Library-owned, zeroed GEMV scratch of the current device for the
// kernel-level entry points (grown on demand; nullptr on failure).
void* op_gemv_scratch(size_t bytes);

template <typename Kern, typename Args>
cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                      const Args& args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

// ---- batched decode state (q_b200_batch_init) -------------------------------------

struct BatchState {
    uint32_t B = 0, TG = 0;        // sequences, groups of 8 in the fragment table
    float* kv = nullptr;           // [B] caches, each [L][n_kv][max_seq][K|V]
    size_t kv_bytes_seq = 0;
    CUtensorMap kv_map;            // attention view: planes (b * L + layer) * n_kv + head
    uint8_t* base = nullptr;       // one allocation for the buffers below
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    uint32_t* frag = nullptr;      // input fragments of the next GEMV
    float* tscale = nullptr;
    float* gath = nullptr;         // tensor parallel: [world][B][v_pad] gathered logits
    StepParams* step = nullptr;    // [B]
    unsigned long long* best = nullptr;
    uint32_t *tok_out = nullptr, *tok_count = nullptr;
    uint32_t tok_cap = 0;
    StepParams* h_step = nullptr;  // pinned [B]
    float wmul = 1.0f, wdiv = 1.0f;  // LM head scale
    // attention launch shape of the batch: with B * n_kv clusters there is
    // parallelism enough for fewer, longer chunks per sequence
    uint32_t att_cs = 0, att_ca = 0, att_slots = 0;
    size_t att_smem = 0;
    // paged caches (q_b200_batch_init_paged): kv is a pool of n_pages pages,
    // each [L][n_kv][page_rows][K|V]; d_pages[b * pages_per_seq + r] is the
    // page holding sequence b's rows [r * page_rows, (r + 1) * page_rows)
    uint32_t page_rows = 0, pages_per_seq = 0, n_pages = 0;
    uint32_t* d_pages = nullptr;
    std::vector<uint32_t> h_pages;     // host mirror, kNoPage where unassigned
    std::vector<uint32_t> free_pages;  // stack of unassigned pages
    bool pages_dirty = false;
    cudaGraphExec_t graph = nullptr;
    uint64_t kernels = 0;
};

// ---- per-context device state ----------------------------------------------------

struct DevState {
    CUtensorMap kv_map;  // tiled-TMA view of this context's KV cache (attention)
    int device = 0;
    // tensor parallelism (q_b200_tp_init before llama_build_graph)
    uint32_t tp_rank = 0, tp_world = 1;
    ncclComm_t comm = nullptr;
    TpShape tp{};
    float* logits_all = nullptr;  // [world * v_pad] gathered logits (world > 1)
    void* peer_buf = nullptr;     // this rank's one-shot all-reduce buffer (IPC-shared)
    TpPeers peers{};
    uint32_t peer_slice = 0;      // floats per slot of the exchange buffer
    bool peers_ready = false;
    cudaStream_t stream = nullptr;
    // tier 3 device twin
    uint8_t* arena = nullptr;
    size_t arena_size = 0, arena_head = 0, arena_base = 0;
    // model (tier 1 in HBM)
    bool built = false;
    q_llama_config cfg{};
    uint32_t hd = 0, kvd = 0;
    uint32_t att_cs = 0, att_ca = 0, att_slots = 0;  // attention cluster size, scores per head, ring
    size_t att_smem = 0;
    std::vector<uint8_t*> qkv, wo, gu, down;
    GemvPlan p_qkv, p_wo, p_gu, p_down;
    ChainPlan cp_first, cp_mid, cp_last;  // [qkv], [wo, gu, down, qkv], [wo, gu, down]
    ChainPlan cp_wo, cp_gu, cp_down;       // one GEMV per launch
    uint32_t chain_phases = 1;
    float* attn_norm = nullptr;  // [L][D]
    float* ffn_norm = nullptr;   // [L][D]
    float* out_norm = nullptr;
    float* embd = nullptr;
    float* out_w = nullptr;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    void* gemv_scratch = nullptr;  // split-slab partial sums + tickets (max over the 4 plans)
    std::vector<void*> weight_allocs;
    // activations (device arena, below the watermark)
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr;
    float* logits = nullptr;
    unsigned long long* best = nullptr;
    uint32_t* chain_bar = nullptr;  // [n_layers][GEMV_MAX_PHASES] grid-barrier counters
    StepParams* step = nullptr;
    uint32_t *tok_out = nullptr, *tok_count = nullptr, *last_tok = nullptr;
    uint32_t tok_cap = 0;
    StepParams* h_step = nullptr;  // pinned, one per row of a call
    // sampling (temperature > 0): parameters, xorshift state, scratch [V]
    SampleParams* samp = nullptr;
    unsigned long long* rng = nullptr;
    float* samp_probs = nullptr;
    uint8_t* samp_keep = nullptr;
    cudaGraphExec_t g_sample = nullptr;  // layers + head + sampler + advance
    BatchState batch;
    // captured graphs (valid for graph_kv)
    void* graph_kv = nullptr;
    cudaGraphExec_t g_body = nullptr, g_full = nullptr;
    uint64_t kernels_body = 0, kernels_full = 0;
    // step tracing: a third graph whose kernels stamp per-kernel times
    cudaGraphExec_t g_trace = nullptr;
    unsigned long long* trace_buf = nullptr;   // [slots][4] device
    unsigned long long* tr_next = nullptr;     // capture cursor (null: untraced)
    uint32_t trace_slots = 0;
    // prompt workspace (allocated on the first prompt of more than one row,
    // grown when a longer prompt comes; never touched by decode steps)
    uint32_t pf_cap = 0;           // rows the workspace holds
    uint8_t* pf_base = nullptr;    // one allocation for all of it
    uint32_t* pf_tok = nullptr;    // [cap] token ids
    float* pf_x = nullptr;         // [cap][D] residual stream
    __half* pf_act = nullptr;      // [2][cap][max(D, H)] activation halves
    float* pf_tscale = nullptr;    // [cap]
    float* pf_q = nullptr;         // [cap][d] rotated queries
    float* pf_o = nullptr;         // [cap][d] attention output
    float* pf_h = nullptr;         // [cap][h] SiLU(gate) * up
    __half* pf_w = nullptr;        // [2][max M][max K] weight halves
    float* pf_rscale = nullptr;    // [max M]
    uint32_t* pf_tok_host = nullptr;  // pinned staging of the prompt ids
};

DevState* state_of(const q_context* ctx, bool create);
void state_erase(const q_context* ctx);
void* dev_arena_alloc(DevState* s, size_t bytes);

q_error_code upload_model(q_context* ctx, DevState* s, const q_llama_model* model);
q_error_code ensure_graphs(q_context* ctx, DevState* s);
q_error_code ensure_sample_graph(q_context* ctx, DevState* s);
q_error_code ensure_sample_scratch(DevState* s);
q_error_code plan_attention(DevState* s);
q_error_code capture_trace_graph(q_context* ctx, DevState* s);
q_error_code check_device_status(const char* where);
// Prompt of seq_len > 1 rows at positions pos.. through the tensor-core
// prefill path (single-GPU contexts); leaves the last row's logits in
// s->logits, its argmax in s->last_tok and the step scalars ready for the
// next decode step.  Asynchronous on s->stream.
q_error_code run_prefill(DevState* s, float* kv, const uint32_t* tokens, uint32_t seq_len, uint32_t pos,
                         bool sample = false);
PFN_cuTensorMapEncodeTiled tensor_map_encoder();
// Reads and clears the device status word of the current device (0 = no
// wait ran out); when it was set, re-zeroes every registered ticket area of
// the device first.
uint32_t take_device_status();
// Ticket / barrier-counter areas that kernels leave zero between launches
// (re-zeroed by take_device_status after a wait ran out).
void register_zero_area(void* p, size_t bytes);
void unregister_zero_area(void* p);
cudaError_t tp_allreduce(DevState* s, void* data, uint32_t n, int op, cudaStream_t st,
                         float* out = nullptr);
void free_model(DevState* s);
void free_batch(DevState* s);

}  // namespace qb200
