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
    t.v_pad = (c.vocab_size + world - 1) / world;
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
