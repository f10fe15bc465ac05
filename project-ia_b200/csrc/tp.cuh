// tp.cuh — tensor parallelism across the GPUs of one node: shard geometry,
// the peer-memory exchange buffers and kernel, and the NCCL entry points the
// decode graph uses.
//
// Rank r of W holds: query heads [r*nh/W, (r+1)*nh/W) and KV heads
// [r*nkv/W, ...) (so the QKV projection and the KV cache are split by head),
// FFN rows [r*H/W, ...) of gate and up, the matching K-slices of wo (its
// heads' columns) and down (its FFN columns), and vocab rows
// [r*ceil(V/W), ...) of the LM head.  wo and down produce partial residual
// updates that an all-reduce sums (fused into the GEMVs over peer memory
// when it is set up, see GemvTp); the argmax key is all-reduced with max.
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

// ---- one-shot all-reduce over peer memory ------------------------------------
// Every rank owns a buffer (shared with the others through CUDA IPC):
//   recv[2][W][slice] fp32 | flags[2][W] u32 | seq u32
// (slice = max(dim, ceil(vocab / W)) floats, a multiple of 4).
// An all-reduce of sequence number q (counted on each rank; every rank runs
// the same sequence) uses parity q & 1: each rank stores its n values into
// recv[q&1][rank] of every rank over NVLink (plain stores, no TMA), fences,
// and sets flags[q&1][rank] = q on every rank (release, system scope); then
// it waits (bounded) until its own flags[q&1][*] >= q and sums the W slices
// in rank order — the same order, so the same bits, on every rank.  Two
// parities suffice: a rank can only reuse a parity after every rank has
// passed the all-reduce in between.
static constexpr uint32_t TP_MAX_RANKS = 8;
// Byte offset of the exchange area the GEMVs use directly (GemvArgs::tp_*):
// word[2][W][slice] u64 (sequence-tagged fp32) | control words (ticket[2] |
// seq[2] | head ticket | key seq | key words, 256 bytes reserved).
inline size_t tp_fused_offset(uint32_t world, uint32_t slice) {
    return ((size_t)2 * world * slice * 4 + (size_t)2 * world * 4 + 256 + 255) / 256 * 256;
}
inline size_t tp_buffer_bytes(uint32_t world, uint32_t slice) {
    return tp_fused_offset(world, slice) + (size_t)2 * world * slice * 8 + 256;
}

struct TpPeers {
    uint8_t* base[TP_MAX_RANKS];  // every rank's buffer, mapped here (own one included)
};

enum TpOp : int { TP_SUM_F32 = 0, TP_MAX_U64 = 1, TP_GATHER_F32 = 2 };

struct TpArgs {
    TpPeers peers;
    void* data;     // in/out: n floats (sum) or one u64 (max); gather: this rank's n floats
    float* out;     // gather: W * n floats, rank order
    uint32_t n, rank, world, op, slice;
};

}  // namespace qb200
