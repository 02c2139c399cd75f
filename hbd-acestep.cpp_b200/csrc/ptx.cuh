// ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers (with bounded waits), 1-D bulk
// async copies (TMA engine, no multicast), and programmatic dependent launch controls.
#pragma once

#include <stdint.h>

namespace acb {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return (uint32_t) __cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and the caller records ACB_DEVERR_TIMEOUT) after `limit`
// unsuccessful polls. Each try_wait blocks for a hardware-defined interval, so the limit
// corresponds to well over a second.
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity, uint32_t limit = (1u << 24)) {
    for (uint32_t i = 0; i < limit; i++) {
        if (mbar_try_wait(bar, parity)) {
            return true;
        }
    }
    return false;
}

// 1-D bulk copy global -> shared through the TMA engine, completing `bytes` of transaction
// count on `bar`. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same with an L2 evict-first policy: streamed weights are read once per pass.
__device__ __forceinline__ void bulk_g2s_stream(void * dst, const void * src, uint32_t bytes, uint64_t * bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Prefetch [src, src + bytes) into L2 (TMA engine; no shared-memory destination). src
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void * src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait until the previous kernel in the stream has completed
// (or triggered), and allow the next kernel to begin launching.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- bounded polling of a word in global memory ----------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// system scope: also sees stores of the host (mapped pinned memory) and of peer GPUs
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Re-reads *word with acquire loads (system scope when SYS) until done(value) holds or limit_ns
// of global time have passed. Returns true when done held; v is the last value read either way.
// Every spin-wait on another agent in this library goes through here, so none can run forever.
template <bool SYS, class Done>
__device__ __forceinline__ bool poll_bounded(const unsigned * word, uint64_t limit_ns, Done done, unsigned & v) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        v = SYS ? ld_acquire_sys(word) : ld_acquire_gpu(word);
        if (done(v)) {
            return true;
        }
        if (globaltimer_ns() - t0 > limit_ns) {
            return false;
        }
    }
}

}  // namespace ptx
}  // namespace acb
