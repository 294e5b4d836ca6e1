// vb_stream.cuh -- PTX helpers for the persistent weight-streaming kernels:
// mbarriers, 1-D TMA bulk copies (cp.async.bulk, no multicast), coherent
// loads, and bounded waits that report a timeout instead of hanging.
#pragma once

#include "vb_common.cuh"

namespace vb {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// src, dst 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 16-byte asynchronous copy global -> shared (no register staging); both
// addresses 16-byte aligned.  Completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// 4-byte asynchronous copy global -> shared (any 4-byte aligned addresses).
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Hint: bring `bytes` (a multiple of 16, 16-byte aligned) of global memory
// into L2 ahead of use.  No completion to wait for.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Acquire-release fence at GPU scope.  After a CTA barrier it also
// releases what other threads of the CTA wrote before the barrier (the
// fence is cumulative), so one thread can publish a whole CTA's results.
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Release-add: the CTA's earlier writes (ordered by a preceding CTA barrier)
// are visible to any thread that acquires the new value.
__device__ __forceinline__ void red_release_gpu(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Named barrier over the consumer warps only (ids 1..15 are free; 0 is
// __syncthreads).
__device__ __forceinline__ void consumer_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Same barrier with an OR-reduction of a per-thread flag: every participant
// gets the same answer, so "any thread saw an error" is a uniform decision
// and no warp can leave a loop that another warp still synchronises in.
__device__ __forceinline__ bool consumer_sync_or(bool v, int nthreads) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred pin, pout;\n"
        " setp.ne.u32 pin, %1, 0;\n"
        " bar.red.or.pred pout, 1, %2, pin;\n"
        " selp.u32 %0, 1, 0, pout;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Spin limit of every wait: about 2 s at 2 GHz, far above any legitimate
// wait; exceeding it records an error code and aborts the kernel cleanly.
constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;

enum StreamError : int {
    STREAM_OK = 0,
    STREAM_TIMEOUT_FULL = 1,    // consumer waited too long for a weight chunk
    STREAM_TIMEOUT_EMPTY = 2,   // producer waited too long for a free slot
    STREAM_TIMEOUT_GRID = 3,    // a grid-wide dependency never completed
    STREAM_BAD_OP = 4,
};

}  // namespace vb
