// api_noalloc.cu — q_b200_gemv_q4_noalloc: the Q4_0 GEMV entry point for
// callers that cannot allocate device memory.
//
// q_b200_gemv_q4 grows a library-owned scratch buffer with cudaMalloc on
// first use (split-slab partial sums and per-slab tickets).  This variant
// takes that scratch from a fixed file-scope device array instead, so a call
// never allocates or frees device memory: usable from code that runs where
// allocation is forbidden or would synchronise (inside allocator hooks,
// real-time loops that must not touch the driver's memory manager, memory
// budgets that are fully reserved up front).
//
// Contract:
//  * the first call on a device (with that device current) resolves the
//    array's address with cudaGetSymbolAddress and sets the kernel's
//    shared-memory attribute; make that first call before any stream
//    capture that should contain the launch;
//  * scratch is kNoAllocScratchBytes; shapes whose plan needs more are
//    rejected with Q_ERR_INVALID_SIZE (the message names both sizes);
//  * the ticket words must be zero before a launch: device globals start
//    zeroed and every launch leaves them zero again; the partial sums need
//    no initial value.  A launch whose bounded wait ran out (a device
//    error, reported by q_b200_device_status) can leave tickets set;
//    q_b200_device_status re-zeroes them (cudaMemset of the array, no
//    allocation), so read it after such an error before the next call;
//  * the address is cached per device for the life of the process: after
//    cudaDeviceReset the process must be restarted before calling again;
//  * one scratch per device: calls that can overlap on the device (other
//    streams, unordered work) race on it and must be serialised by the
//    caller.
#include <mutex>

namespace qb200 {

static constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
struct NoAllocDevice {
    std::once_flag once;
    void* scratch = nullptr;
    cudaError_t err = cudaSuccess;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
}  // namespace

}  // namespace qb200

using namespace qb200;

extern "C" q_error_code q_b200_gemv_q4_noalloc(const void* d_packed, uint32_t M, uint32_t K,
                                               const float* d_x, float* d_y, void* stream) {
    if (!d_packed || !d_x || !d_y) return Q_ERR_INVALID_ARG;
    if (d_x == d_y) return Q_ERR_ALIASING;
    if (((uintptr_t)d_x & 15) || ((uintptr_t)d_packed & 15)) return Q_ERR_MISALIGNED;
    GemvPlan p;
    ChainPlan cp;
    if (!plan_single(M, K, p, cp)) return Q_ERR_INVALID_SIZE;
    if (cp.scratch_bytes() > kNoAllocScratchBytes) {
        const std::string where = "q_b200_gemv_q4_noalloc: M=" + std::to_string(M) +
                                  " K=" + std::to_string(K) + " needs " +
                                  std::to_string(cp.scratch_bytes()) + " scratch bytes, limit " +
                                  std::to_string(kNoAllocScratchBytes);
        set_last_error(where.c_str(), cudaErrorInvalidValue);
        return Q_ERR_INVALID_SIZE;
    }
    int dev = 0;
    Q_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices) return Q_ERR_INVALID_ARG;
    NoAllocDevice& d = g_noalloc_dev[dev];
    std::call_once(d.once, [&d] {
        d.err = cudaGetSymbolAddress(&d.scratch, g_noalloc_scratch);
        if (d.err == cudaSuccess) register_zero_area(d.scratch, ChainPlan::kTicketWords * 4);
        if (d.err == cudaSuccess) d.err = ensure_smem_attr((const void*)q4_slab_kernel<false>, 227 * 1024);
    });
    Q_CUDA(d.err);
    GemvArgs a{};
    a.w = (const uint8_t*)d_packed;
    a.x = d_x;
    a.y = d_y;
    a.epi = EPI_STORE;
    Q_CUDA(launch_single(cp, p, a, d.scratch, (cudaStream_t)stream));
    return Q_OK;
}
