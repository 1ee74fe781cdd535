// Device-side helpers shared by the sm_100a kernels of the k200 matmul path:
// shared-memory addressing, mbarriers, 1-D bulk (TMA) copies, bounded waits
// and the per-device error word.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace k200 {

// Error codes a kernel may post into the per-device error word (mapped host
// memory, read by kunlun::wait()).  Kernels never trap: a wait that runs out
// of its iteration budget records its code and the kernel returns early.
enum KernelError : int {
    kErrNone = 0,
    kErrBulkTimeout = 0x4b01,   // a bulk copy never completed its mbarrier phase
    kErrMmaTimeout = 0x4b02,    // a tcgen05 commit never arrived
    kErrPeerTimeout = 0x4b03,   // a peer flag never arrived
};

// Budget for one mbarrier wait, in try_wait attempts.
constexpr uint32_t kWaitBudget = 1u << 19;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// `count` arrivals at once.
__device__ __forceinline__ void mbar_arrive_count(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// One potentially blocking test of an mbarrier phase: a thread whose phase
// is not complete is suspended until it completes or about kSuspendNs pass,
// so waiting warps do not take issue slots from working ones.
constexpr uint32_t kSuspendNs = 2000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and posts `code`) when
// the budget runs out (at most kWaitBudget suspensions, about a second).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    for (uint32_t i = 0; i < kWaitBudget; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, code);
    return false;
}

// The same bounded wait for a thread whose wait is not on the critical path
// (a producer with many stages of slack): between tests it sleeps `sleep_ns`,
// so a long wait does not take issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, int *err, int code,
                                                unsigned sleep_ns) {
    for (uint32_t i = 0; i < kWaitBudget; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(sleep_ns);
    }
    if (err) atomicExch(err, code);
    return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 eviction-first hint: streamed weights are read once.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: let the next kernel on the stream start its
// prologue, and wait for the previous kernel's memory before touching it.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Packed f32x2 arithmetic (sm_100a): one instruction, two IEEE f32 results.
// Pairs are formed and split with PTX vector moves, which the register
// allocator resolves to an aligned register pair (no instructions).
__device__ __forceinline__ unsigned long long u2_pack(uint32_t lo, uint32_t hi) {
    unsigned long long v;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo), "r"(hi));
    return v;
}
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    return u2_pack(__float_as_uint(lo), __float_as_uint(hi));
}
__device__ __forceinline__ float f2_lo(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
// lo + hi of a pair
__device__ __forceinline__ float f2_sum(unsigned long long v) {
    uint32_t lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
    return __uint_as_float(lo) + __uint_as_float(hi);
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// binary16 bits -> binary32, exact (subnormals, Inf and NaN preserved).
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace k200
