// tp.cuh — tensor parallelism across the GPUs of one node: shard geometry
// and the NCCL entry points the decode graph uses.
//
// Rank r of W holds: query heads [r*nh/W, (r+1)*nh/W) and KV heads
// [r*nkv/W, ...) (so the QKV projection and the KV cache are split by head),
// FFN rows [r*H/W, ...) of gate and up, the matching K-slices of wo (its
// heads' columns) and down (its FFN columns), and vocab rows
// [r*ceil(V/W), ...) of the LM head.  wo and down produce partial residual
// updates that an all-reduce sums; the argmax key is all-reduced with max.
// Norm gains, RoPE tables and the embedding are replicated.
//
// NCCL is opened at run time (dlopen of libnccl.so.2) so the library binds
// to whichever NCCL the process already uses (e.g. the one torch loaded).
#pragma once

#include <nccl.h>

#include <cstdint>

#include "qorus_types.h"

namespace qb200 {

struct TpShape {
    uint32_t rank = 0, world = 1;
    uint32_t nh, nkv;        // local query / KV heads
    uint32_t d, kvd;         // local q width (nh*hd) and k/v width (nkv*hd)
    uint32_t q0, kv0;        // first global q row / k-v row of this rank
    uint32_t h, h0;          // local FFN width and first FFN row
    uint32_t v, v0, v_pad;   // local vocab rows, first vocab row, rows per rank (ceil)
};

// Shard geometry of `rank` in `world`; false when the model does not split
// evenly (heads, KV heads, or FFN width by 32*world).
bool tp_shape(const q_llama_config& c, uint32_t rank, uint32_t world, TpShape& t);

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char* (*error_string)(ncclResult_t);
};

// The process's NCCL (nullptr, with the last error set, when unavailable).
const NcclApi* nccl();

}  // namespace qb200
