// tp.cu — shard geometry, the run-time NCCL binding, and the additive
// tensor-parallel entry points q_b200_tp_unique_id / q_b200_tp_init.
#include <dlfcn.h>

#include <mutex>

#include "runtime.cuh"
#include "tp.cuh"

namespace qb200 {

bool tp_shape(const q_llama_config& c, uint32_t rank, uint32_t world, TpShape& t) {
    if (world == 0 || rank >= world) return false;
    if (c.n_heads % world || c.n_kv_heads % world || c.hidden_dim % (32 * world)) return false;
    const uint32_t hd = c.dim / c.n_heads;
    t.rank = rank;
    t.world = world;
    t.nh = c.n_heads / world;
    t.nkv = c.n_kv_heads / world;
    t.d = t.nh * hd;
    t.kvd = t.nkv * hd;
    if (t.d % 32) return false;  // wo's K-slice is whole Q4_0 blocks
    t.q0 = rank * t.d;
    t.kv0 = rank * t.kvd;
    t.h = c.hidden_dim / world;
    t.h0 = rank * t.h;
    t.v_pad = ((c.vocab_size + world - 1) / world + 3) / 4 * 4;  // a multiple of 4 (float4 gathers)
    t.v0 = std::min(c.vocab_size, rank * t.v_pad);
    t.v = std::min(c.vocab_size, t.v0 + t.v_pad) - t.v0;
    return true;
}

const NcclApi* nccl() {
    static NcclApi api{};
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
        ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce &&
             api.all_gather && api.error_string;
    });
    if (!ok) set_last_error("libnccl.so.2 not loadable", cudaErrorSharedObjectInitFailed);
    return ok ? &api : nullptr;
}

// ---- peer-memory all-reduce kernel ----------------------------------------------


__global__ void __launch_bounds__(512) tp_allreduce_kernel(const TpArgs a) {
    constexpr uint32_t T = 512;
    const uint32_t tid = threadIdx.x, W = a.world, me = a.rank;
    __shared__ uint32_t seq;
    pdl_trigger();  // the next kernel may start streaming its weights
    pdl_wait();     // the input is the previous kernel's output
    uint8_t* mine = a.peers.base[me];
    const size_t slice = (size_t)a.slice * 4;
    uint32_t* myflags = reinterpret_cast<uint32_t*>(mine + 2 * W * slice);
    uint32_t* seqp = myflags + 2 * W;
    if (tid == 0) seq = *seqp + 1;
    __syncthreads();
    const uint32_t q = seq, par = q & 1;
    // 1. this rank's values into slot [par][me] of every rank
    if (a.op != TP_MAX_U64) {
        const float4* src = reinterpret_cast<const float4*>(a.data);
        const uint32_t n4 = a.n / 4;
        for (uint32_t r = 0; r < W; ++r) {
            float4* dst = reinterpret_cast<float4*>(a.peers.base[r] + ((size_t)par * W + me) * slice);
            for (uint32_t i = tid; i < n4; i += T) dst[i] = __ldcg(src + i);
        }
    } else if (tid < W) {
        *reinterpret_cast<unsigned long long*>(a.peers.base[tid] + ((size_t)par * W + me) * slice) =
            *reinterpret_cast<const unsigned long long*>(a.data);
    }
    __syncthreads();
    if (tid < W) {
        __threadfence_system();
        uint32_t* f = reinterpret_cast<uint32_t*>(a.peers.base[tid] + 2 * W * slice) + par * W + me;
        st_release_sys(f, q);
    }
    // 2. every rank's slice has arrived here
    if (tid < W) {
        const unsigned long long t0 = gtimer(), lim = qdev_wait_ns();
        while (ld_acquire_sys(myflags + par * W + tid) < q) {
            if (gtimer() - t0 > lim) {
                qdev_fail(QDEV_PEER_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
    // 3. reduce in rank order
    if (a.op == TP_SUM_F32) {
        float4* out = reinterpret_cast<float4*>(a.data);
        const uint32_t n4 = a.n / 4;
        for (uint32_t i = tid; i < n4; i += T) {
            float4 acc = __ldcg(reinterpret_cast<const float4*>(mine + ((size_t)par * W) * slice) + i);
            for (uint32_t r = 1; r < W; ++r) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(mine + ((size_t)par * W + r) * slice) + i);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            out[i] = acc;
        }
    } else if (a.op == TP_GATHER_F32) {
        const uint32_t n4 = a.n / 4;
        for (uint32_t r = 0; r < W; ++r) {
            const float4* src = reinterpret_cast<const float4*>(mine + ((size_t)par * W + r) * slice);
            float4* dst = reinterpret_cast<float4*>(a.out + (size_t)r * a.n);
            for (uint32_t i = tid; i < n4; i += T) dst[i] = __ldcg(src + i);
        }
    } else if (tid == 0) {
        unsigned long long m = 0;
        for (uint32_t r = 0; r < W; ++r) {
            const unsigned long long v =
                __ldcg(reinterpret_cast<const unsigned long long*>(mine + ((size_t)par * W + r) * slice));
            m = v > m ? v : m;
        }
        *reinterpret_cast<unsigned long long*>(a.data) = m;
    }
    if (tid == 0) *seqp = q;
}

cudaError_t tp_allreduce(DevState* s, void* data, uint32_t n, int op, cudaStream_t st, float* out) {
    if (n > s->peer_slice || (op != TP_MAX_U64 && n % 4)) return cudaErrorInvalidValue;
    TpArgs a{};
    a.peers = s->peers;
    a.data = data;
    a.out = out;
    a.slice = s->peer_slice;
    a.n = n;
    a.rank = s->tp_rank;
    a.world = s->tp_world;
    a.op = (uint32_t)op;
    return launch_ex(tp_allreduce_kernel, dim3(1), dim3(512), 0, st, true, a);
}

}  // namespace qb200

using namespace qb200;

extern "C" {

q_error_code q_b200_tp_unique_id(void* id, size_t bytes) {
    if (!id || bytes < sizeof(ncclUniqueId)) return Q_ERR_INVALID_ARG;
    const NcclApi* n = nccl();
    if (!n) return Q_ERR_INVALID_ARG;
    ncclUniqueId u;
    const ncclResult_t r = n->get_unique_id(&u);
    if (r != ncclSuccess) {
        set_last_error(n->error_string(r), cudaErrorUnknown);
        return Q_ERR_INVALID_ARG;
    }
    std::memcpy(id, &u, sizeof u);
    return Q_OK;
}

q_error_code q_b200_tp_init(q_context* ctx, uint32_t rank, uint32_t world, const void* id, size_t bytes) {
    if (!ctx || !id || bytes < sizeof(ncclUniqueId) || world == 0 || rank >= world) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, true);
    if (!s) return Q_ERR_ALLOC_FAILED;
    if (s->built || s->comm) return Q_ERR_INVALID_ARG;  // before llama_build_graph, once
    if (world > 1) {
        const NcclApi* n = nccl();
        if (!n) return Q_ERR_INVALID_ARG;
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof u);
        ncclComm_t comm = nullptr;
        const ncclResult_t r = n->comm_init_rank(&comm, (int)world, u, (int)rank);
        if (r != ncclSuccess) {
            set_last_error(n->error_string(r), cudaErrorUnknown);
            return Q_ERR_INVALID_ARG;
        }
        s->comm = comm;
    }
    s->tp_rank = rank;
    s->tp_world = world;
    return Q_OK;
}

// IPC handle of this rank's peer buffer (allocated here on first call).
q_error_code q_b200_tp_ipc_handle(q_context* ctx, void* out, size_t bytes) {
    if (!ctx || !out || bytes < sizeof(cudaIpcMemHandle_t)) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, false);
    if (!s || s->tp_world < 2 || s->tp_world > TP_MAX_RANKS) return Q_ERR_INVALID_ARG;
    if (!s->peer_buf) {
        const q_model_header* hd = ctx->header;
        if (!hd) return Q_ERR_INVALID_ARG;  // after q_init_memory: sized from the model header
        const uint32_t vpad = ((hd->vocab_size + s->tp_world - 1) / s->tp_world + 3) / 4 * 4;
        s->peer_slice = (std::max(hd->dim, vpad) + 3) / 4 * 4;
        const size_t nb = tp_buffer_bytes(s->tp_world, s->peer_slice);
        Q_CUDA(dev_malloc(&s->peer_buf, nb));
        Q_CUDA(cudaMemset(s->peer_buf, 0, nb));
        Q_CUDA(cudaDeviceSynchronize());
    }
    cudaIpcMemHandle_t h;
    Q_CUDA(cudaIpcGetMemHandle(&h, s->peer_buf));
    std::memcpy(out, &h, sizeof h);
    return Q_OK;
}

// Map every rank's buffer (handles in rank order, world * 64 bytes); from
// then on the decode graph all-reduces over peer memory instead of NCCL.
q_error_code q_b200_tp_ipc_open(q_context* ctx, const void* handles, size_t bytes) {
    if (!ctx || !handles) return Q_ERR_INVALID_ARG;
    DevState* s = state_of(ctx, false);
    if (!s || !s->peer_buf || s->built) return Q_ERR_INVALID_ARG;
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    if (bytes < s->tp_world * hb) return Q_ERR_INVALID_ARG;
    for (uint32_t r = 0; r < s->tp_world; ++r) {
        if (r == s->tp_rank) {
            s->peers.base[r] = (uint8_t*)s->peer_buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, (const uint8_t*)handles + r * hb, hb);
        void* p = nullptr;
        Q_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        s->peers.base[r] = (uint8_t*)p;
    }
    s->peers_ready = true;
    return Q_OK;
}

q_error_code q_b200_tp_shape(const q_llama_config* cfg, uint32_t rank, uint32_t world, uint32_t* out,
                             uint32_t n) {
    if (!cfg || !out || n < 13) return Q_ERR_INVALID_ARG;
    TpShape t;
    if (!tp_shape(*cfg, rank, world, t)) return Q_ERR_INVALID_CONFIG;
    const uint32_t v[13] = {t.rank, t.world, t.nh, t.nkv, t.d, t.kvd, t.q0, t.kv0, t.h, t.h0, t.v, t.v0, t.v_pad};
    std::memcpy(out, v, sizeof v);
    return Q_OK;
}

}  // extern "C"
