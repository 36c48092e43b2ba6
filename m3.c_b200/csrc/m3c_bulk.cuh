// Shared-memory pipelines of the sm_100a kernels: mbarriers, bounded waits
// and 1-D TMA bulk copies (cp.async.bulk global -> shared with mbarrier
// completion; no tensor map, no multicast).  Every wait gives up after
// BULK_WAIT_NS and reports it, so a kernel whose partner never arrives ends
// with an error status instead of hanging the GPU.

#pragma once

#include <cstdint>

#include "m3c_kernels.h"

namespace m3c {

constexpr uint64_t BULK_WAIT_NS = 2000000000ull;  // 2 s per wait, then give up
constexpr uint32_t BULK_TIMEOUT_CODE = 9u;        // M3_STATUS_INTERNAL

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 state;\n\tmbarrier.arrive.shared::cta.b64 state, [%0];\n\t}" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// One arrival that also expects `bytes` of copies to complete on the phase.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 state;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 state, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t now_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for the phase of `parity` to complete; false after BULK_WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
    const uint32_t addr = smem_addr(bar);
    uint64_t deadline = 0;
    for (uint32_t spin = 0;; ++spin) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((spin & 255u) == 0u) {
            const uint64_t t = now_ns();
            if (deadline == 0) {
                deadline = t + BULK_WAIT_NS;
            } else if (t > deadline) {
                return false;
            }
        }
    }
}

// Poll a shared-memory word with acquire loads until it equals `want`
// (false after BULK_WAIT_NS): what its writer stored before its release
// is then visible.
__device__ __forceinline__ bool poll_acquire(volatile int *word, int want)
{
    const uint32_t addr = smem_addr(const_cast<int *>(word));
    uint64_t deadline = 0;
    for (uint32_t spin = 0;; ++spin) {
        int seen;
        asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(seen) : "r"(addr) : "memory");
        if (seen == want) return true;
        if ((spin & 255u) == 0u) {
            const uint64_t t = now_ns();
            if (deadline == 0) {
                deadline = t + BULK_WAIT_NS;
            } else if (t > deadline) {
                return false;
            }
        }
    }
}

// Copy `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global to shared memory; completion counts on `bar`.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// A wait that gave up: the launch's first command fails with an internal
// error.
__device__ __forceinline__ void bulk_timed_out(m3c_status *status, uint32_t command)
{
    atomicMin(&status->fail_command, command);
    atomicExch(&status->fail_code, BULK_TIMEOUT_CODE);
}

}  // namespace m3c
