// api.cu — the upstream memory-tier API (include/qorus.h) served on a B200.
//
// Memory tiers follow upstream src/core/memory.c:60-355: tier 1 is still
// the read-only mmap of the model file (the one-time upload source), tier 2
// (KV) is HBM, tier 3 is the host bump arena for views plus a device twin
// for activations.  Return codes and validation order are upstream's.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdlib>

#include "runtime.cuh"

using namespace qb200;

static size_t align64(size_t n) { return (n + 63) & ~(size_t)63; }

extern "C" {

// ---- tier 1 -------------------------------------------------------------------

q_error_code q_init_memory_ex(q_context* ctx, const char* path, q_mmap_strategy strategy) {
    if (!ctx || !path) return Q_ERR_INVALID_ARG;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return Q_ERR_FILE_OPEN;
    struct stat st;
    if (fstat(fd, &st) < 0) {
        close(fd);
        return Q_ERR_FILE_STAT;
    }
    const size_t size = (size_t)st.st_size;
    if (size < Q_HEADER_SIZE) {
        close(fd);
        return Q_ERR_FILE_TOO_SMALL;
    }
    int flags = MAP_PRIVATE;
    if (strategy == Q_MMAP_EAGER) flags |= MAP_POPULATE;
    void* m = mmap(nullptr, size, PROT_READ, flags, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return Q_ERR_MMAP_FAILED;
    madvise(m, size, MADV_SEQUENTIAL | MADV_WILLNEED);
    q_model_header* h = (q_model_header*)m;
    if (h->magic != Q_MAGIC) {
        munmap(m, size);
        return Q_ERR_INVALID_MAGIC;
    }
    ctx->weights_mmap = m;
    ctx->weights_size = size;
    ctx->header = h;
    return Q_OK;
}

q_error_code q_init_memory(q_context* ctx, const char* path) {
    return q_init_memory_ex(ctx, path, Q_MMAP_LAZY);
}

// ---- tier 2 -------------------------------------------------------------------

q_error_code q_alloc_kv_cache(q_context* ctx, size_t kv_size) {
    if (!ctx) return Q_ERR_INVALID_ARG;
    if (ctx->kv_buffer) return Q_ERR_INVALID_ARG;
    if (kv_size > SIZE_MAX - 63) return Q_ERR_OVERFLOW;
    const size_t a = align64(kv_size);
    if (a == 0) return Q_ERR_OVERFLOW;
    DevState* s = state_of(ctx, true);
    if (!s) return Q_ERR_ALLOC_FAILED;
    void* p = nullptr;
    if (!cuda_ok(dev_malloc(&p, a), "dev_malloc(kv)")) return Q_ERR_ALLOC_FAILED;
    if (!cuda_ok(cudaMemset(p, 0, a), "cudaMemset(kv)")) {
        cudaFree(p);
        return Q_ERR_ALLOC_FAILED;
    }
    ctx->kv_buffer = p;
    ctx->kv_size = a;
    return Q_OK;
}

// ---- tier 3 -------------------------------------------------------------------

q_error_code q_alloc_arena(q_context* ctx, size_t arena_size) {
    if (!ctx) return Q_ERR_INVALID_ARG;
    if (ctx->scratch_buffer) return Q_ERR_INVALID_ARG;
    if (arena_size > SIZE_MAX - 63) return Q_ERR_OVERFLOW;
    const size_t a = align64(arena_size);
    if (a == 0) return Q_ERR_OVERFLOW;
    DevState* s = state_of(ctx, true);
    if (!s) return Q_ERR_ALLOC_FAILED;
    void* h = aligned_alloc(Q_ALIGN, a);
    if (!h) return Q_ERR_ALLOC_FAILED;
    void* d = nullptr;
    if (!cuda_ok(dev_malloc(&d, a), "dev_malloc(arena)")) {
        free(h);
        return Q_ERR_ALLOC_FAILED;
    }
    s->arena = (uint8_t*)d;
    s->arena_size = a;
    s->arena_head = s->arena_base = 0;
    ctx->scratch_buffer = h;
    ctx->scratch_size = a;
    ctx->scratch_head = 0;
    ctx->scratch_base_offset = 0;
    return Q_OK;
}

void* q_arena_alloc(q_context* ctx, size_t size) {
    if (!ctx || !ctx->scratch_buffer) return nullptr;
    if (size > SIZE_MAX - 63) return nullptr;
    const size_t a = align64(size);
    if (a == 0) return nullptr;
    if (ctx->scratch_head > SIZE_MAX - a) return nullptr;
    const size_t nh = ctx->scratch_head + a;
    if (nh > ctx->scratch_size) return nullptr;
    void* p = (uint8_t*)ctx->scratch_buffer + ctx->scratch_head;
    ctx->scratch_head = nh;
    return p;
}

void q_arena_reset(q_context* ctx) {
    if (!ctx) return;
    ctx->scratch_head = ctx->scratch_base_offset;
    if (DevState* s = state_of(ctx, false)) s->arena_head = s->arena_base;
}

void q_free_memory(q_context* ctx) {
    if (!ctx) return;
    state_erase(ctx);  // device arena, weights, graphs, stream
    if (ctx->scratch_buffer) {
        free(ctx->scratch_buffer);
        ctx->scratch_buffer = nullptr;
        ctx->scratch_size = ctx->scratch_head = ctx->scratch_base_offset = 0;
    }
    if (ctx->kv_buffer) {
        cudaFree(ctx->kv_buffer);
        ctx->kv_buffer = nullptr;
        ctx->kv_size = 0;
    }
    if (ctx->weights_mmap) {
        munmap(ctx->weights_mmap, ctx->weights_size);
        ctx->weights_mmap = nullptr;
        ctx->weights_size = 0;
        ctx->header = nullptr;
    }
}

const char* q_strerror(q_error_code err) {
    switch (err) {
        case Q_OK: return "Success";
        case Q_ERR_NULL_PTR: return "Null pointer argument";
        case Q_ERR_FILE_OPEN: return "Failed to open file";
        case Q_ERR_FILE_STAT: return "Failed to stat file";
        case Q_ERR_FILE_TOO_SMALL: return "File too small (corrupt header?)";
        case Q_ERR_MMAP_FAILED: return "mmap() failed";
        case Q_ERR_INVALID_MAGIC: return "Invalid file magic (not a Qorus file)";
        case Q_ERR_ALLOC_FAILED: return "Memory allocation failed";
        case Q_ERR_ARENA_OOM: return "Arena Out of Memory";
        case Q_ERR_INVALID_CONFIG: return "Invalid model configuration";
        case Q_ERR_INVALID_ARG: return "Invalid argument";
        case Q_ERR_ALIASING: return "Input/output aliasing detected";
        case Q_ERR_OVERFLOW: return "Integer overflow detected";
        case Q_ERR_MISALIGNED: return "Pointer not properly aligned";
        case Q_ERR_INVALID_DTYPE: return "Invalid data type";
        case Q_ERR_INVALID_SIZE: return "Invalid size";
        default: return "Unknown error";
    }
}

const char* q_b200_last_error(void) { return last_error_cstr(); }
uint64_t q_b200_kernel_launches(void) { return g_kernel_launches.load(); }

uint64_t q_b200_device_allocations(void) { return g_device_allocs.load(); }

}  // extern "C"
