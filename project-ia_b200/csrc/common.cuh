// common.cuh — shared device helpers for the sm_100a kernels of libqorus_b200.
//
// Inline-PTX wrappers for the Blackwell features the kernels use: mbarrier
// (transaction-count barriers), cp.async.bulk (the 1-D TMA engine: global ->
// shared copies that complete on an mbarrier), programmatic dependent launch
// (griddepcontrol) and streaming loads.  Every spin wait is bounded: after
// g_qdev_wait_ns of wall time (2 s unless the host sets it, see
// q_b200_set_wait_limit_ns) or Q_SPIN_LIMIT polls it records an error code in
// the device status word and gives up, so a lost transaction never hangs the
// GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifndef Q_SPIN_LIMIT
#define Q_SPIN_LIMIT (1u << 26)
#endif

// Device status word (one per library load); 0 = OK.  Kernels write a code
// here when a bounded wait times out; the host reads it after sync.
enum : uint32_t {
    QDEV_OK = 0,
    QDEV_WAIT_FULL_TIMEOUT = 1,
    QDEV_WAIT_EMPTY_TIMEOUT = 2,
    QDEV_COMBINE_TIMEOUT = 3,
    QDEV_BAD_ARG = 4,
    QDEV_GRID_TIMEOUT = 5,
    QDEV_PEER_TIMEOUT = 6,
};

// The library is one translation unit (csrc/libqorus_b200.cu), so the
// status word is defined here.
__device__ uint32_t g_qdev_status = 0;

__device__ __forceinline__ void qdev_fail(uint32_t code) { atomicCAS(&g_qdev_status, 0u, code); }

// Wall-time limit of every bounded wait, in ns (one per device; the host
// may lower it, e.g. so a test can make a wait run out quickly).
__device__ unsigned long long g_qdev_wait_ns = 2000000000ull;
__device__ __forceinline__ unsigned long long qdev_wait_ns() {
    return *reinterpret_cast<volatile unsigned long long*>(&g_qdev_wait_ns);
}

// Global nanosecond timer (bounds every wait in wall time).
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes or about `ns` nanoseconds pass, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false (and an error code) after
// g_qdev_wait_ns of wall time or Q_SPIN_LIMIT polls, whichever comes first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer(), lim = qdev_wait_ns();
    for (uint32_t i = 0; i < Q_SPIN_LIMIT; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 20000)) return true;
        if (gtimer() - t0 > lim) break;
    }
    qdev_fail(code);
    return false;
}

// ---- system-scope flags (tensor-parallel peers over NVLink) ------------------

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- 1-D bulk copy (TMA engine) -------------------------------------------
// Both addresses 16-byte aligned, size a multiple of 16 (checked by callers).
// Source is always this GPU's own memory; no multicast.

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---- programmatic dependent launch ------------------------------------------

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- step tracing ---------------------------------------------------------------
// A traced kernel gets a slot of 4 u64: [0] earliest CTA entry, [1] earliest
// end of the programmatic-dependency wait, [2] latest exit (ns, %globaltimer).
// Slots start as {~0, ~0, 0, 0}; a null slot disables tracing (one branch).

__device__ __forceinline__ void trace_mark(unsigned long long* slot, int which) {
    if (slot == nullptr) return;
    if (which < 2) atomicMin(slot + which, gtimer());
    else atomicMax(slot + 2, gtimer());
}

// ---- loads / misc -------------------------------------------------------------

__device__ __forceinline__ float4 ldg_stream_f4(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Upstream polynomial exp (src/ops/avx2/avx_math.h:10-61): degree-5 Taylor
// polynomial by Horner with FMA on x clamped to [-5,5], floored at 0;
// x < -10 gives 0, x > 10 gives 22026.  This is the upstream project's own
// approximation, restated so device results match it bit for bit.
__device__ __forceinline__ float exp_poly(float x) {
    if (x < -10.0f) return 0.0f;
    if (x > 10.0f) return 22026.0f;
    float c = x < 5.0f ? x : 5.0f;
    c = c > -5.0f ? c : -5.0f;
    float r = 0.00833333f;
    r = __fmaf_rn(r, c, 0.04166667f);
    r = __fmaf_rn(r, c, 0.16666667f);
    r = __fmaf_rn(r, c, 0.5f);
    r = __fmaf_rn(r, c, 1.0f);
    r = __fmaf_rn(r, c, 1.0f);
    return r > 0.0f ? r : 0.0f;
}

// x * sigmoid(x) the way upstream's vector body computes it
// (src/ops/avx2/silu.c:60-80): 1 / (1 + exp_poly(-x)), then x * that.
__device__ __forceinline__ float silu_poly(float x) {
    float d = __fadd_rn(1.0f, exp_poly(-x));
    float sg = __fdiv_rn(1.0f, d);
    return __fmul_rn(x, sg);
}
