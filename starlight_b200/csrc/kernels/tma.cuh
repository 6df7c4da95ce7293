// Bulk asynchronous copies (the TMA unit's 1-D form, cp.async.bulk) into
// shared memory, completed on an mbarrier, with bounded waits.
//
// No multicast anywhere: every copy reads this GPU's own memory into this
// CTA's shared memory. Copies need 16-byte aligned addresses and sizes that
// are multiples of 16 bytes; callers check this on the host.
#pragma once

#include <stdint.h>

namespace slc {

// Error codes written to the device error word.
enum DeviceErrorCode : uint32_t {
    kErrNone = 0,
    kErrGatherId = 1,      // gather id out of range (host checks first)
    kErrWaitTimeout = 2,   // an mbarrier wait gave up
    kErrBadScalar = 3,     // a device-resident scalar failed its bounds check
};

// Records an error for the host (pinned, mapped host word; plain store).
__device__ __forceinline__ void report_error(uint32_t *flag, uint32_t code) {
    if (flag) *reinterpret_cast<volatile uint32_t *>(flag) = code;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most `limit_ns`
// nanoseconds of wall time. Returns false when the limit is reached (after
// recording kErrWaitTimeout and raising the CTA's abort word, so that the
// CTA's other waits give up at once) or when the abort word is already set.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err,
                                          volatile int *abort,
                                          uint64_t limit_ns = 1000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_ns() - t0 > limit_ns) {
            report_error(err, kErrWaitTimeout);
            *abort = 1;
            return false;
        }
    }
}

// L2 policy for data read exactly once (weights, KV rows).
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// One bulk copy global -> shared, completing `bytes` of transaction count on
// `bar`. dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Tiled 2-D tensor copy global -> shared through a tensor map (a
// __grid_constant__ kernel parameter), completing `bytes` of the box on
// `bar`. The innermost coordinate x times the element size must be a
// multiple of 16 bytes (checked by the callers).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y,
                                            uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Tiled 2-D tensor copy global -> shared without a cache hint.
__device__ __forceinline__ void tma_load_2d_nohint(void *dst, const void *tmap, int x, int y,
                                                   uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// 4-byte asynchronous copy global -> shared (LDGSTS).
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
}

// Makes `bar` track this thread's prior cp.async copies: its current phase
// cannot complete before they land (net-zero change of the pending count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

}  // namespace slc
