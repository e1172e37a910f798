// nsc_tma.cuh -- TMA (cp.async.bulk.tensor) and mbarrier helpers for the
// tiled sm_100a kernels, plus the host-side tensor-map encoder.
//
// No load here uses cluster multicast: every tensor copy reads this GPU's
// own memory into this CTA's shared memory.  Every wait on an mbarrier is
// bounded (kSleepWaits hinted waits); a wait that gives up bumps a device counter
// (see wait_timeout_counter) and the caller unwinds instead of hanging.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace nsc {


__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\t"
                 "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\t"
                 "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a waiting warp is parked by the
// hardware until the phase completes or the hint (1 ms) expires, instead of
// spinning and taking issue slots from the warps that compute.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
                 : "memory");
    return ok != 0;
}

// The same waits by 32-bit shared address (no generic-to-shared conversion).
__device__ __forceinline__ bool mbar_try_wait32(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait_sleep32(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive32(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\t"
                 "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
                 : "memory");
}

// Bounded wait for the phase of `parity` to complete: at most
// kSleepWaits hinted waits (seconds in total).  Returns false (and counts a
// timeout) when the budget runs out.
constexpr uint32_t kSleepWaits = 4096;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned int* timeouts,
                                          uint32_t budget = kSleepWaits) {
    if (mbar_try_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < budget; ++i)
        if (mbar_try_wait_sleep(bar, parity)) return true;
    atomicAdd(timeouts, 1u);
    return false;
}
// As mbar_wait32, but a CTA-wide abort flag (shared memory) is checked
// before any suspension: once one thread gave up, the others return at once
// instead of each running out its own limit.  The fast path (phase already
// complete) is a single try_wait.
// abort_flag[1] holds the wait budget (hinted sleeps) of the launch.
static __device__ __noinline__ bool mbar_wait32_slow(uint32_t bar, uint32_t parity,
                                              unsigned int* timeouts,
                                              volatile int* abort_flag) {
    if (*abort_flag) return false;
    const uint32_t budget = static_cast<uint32_t>(abort_flag[1]);
    for (uint32_t i = 0; i < budget; ++i) {
        if (mbar_try_wait_sleep32(bar, parity)) return true;
        if ((i & 63u) == 63u && *abort_flag) return false;
    }
    atomicAdd(timeouts, 1u);
    *abort_flag = 1;
    return false;
}
__device__ __forceinline__ bool mbar_wait32_ab(uint32_t bar, uint32_t parity,
                                               unsigned int* timeouts,
                                               volatile int* abort_flag) {
    if (mbar_try_wait32(bar, parity)) return true;
    return mbar_wait32_slow(bar, parity, timeouts, abort_flag);
}
__device__ __forceinline__ bool mbar_wait32(uint32_t bar, uint32_t parity,
                                            unsigned int* timeouts) {
    if (mbar_try_wait32(bar, parity)) return true;
    for (uint32_t i = 0; i < kSleepWaits; ++i)
        if (mbar_try_wait_sleep32(bar, parity)) return true;
    atomicAdd(timeouts, 1u);
    return false;
}

// 3-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
        "r"(c2)
        : "memory");
}

// 4-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2, int32_t c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
        "r"(c2), "r"(c3)
        : "memory");
}

// Named barrier over `count` threads (id 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Host: device address of the wait-timeout counter of the current device
// (nullptr on failure, with the error recorded).
unsigned int* wait_timeout_counter();

// Host: the wait budget (hinted sleeps) and the test hook's skipped copy
// index (-1: none) the next tiled launch uses (set by nsc_test_wait_fault).
void wait_fault_settings(int* skip_copy, unsigned* budget);

// Host: encode a 3-D tensor map {W, H, planes} with box {bw, bh, 1}.
// Returns false with a message in `err` when the driver refuses.
bool encode_map_3d(CUtensorMap* map, const void* base, int elem_bytes,
                   CUtensorMapDataType dtype, uint64_t W, uint64_t H,
                   uint64_t planes, uint32_t bw, uint32_t bh, const char** err);

// Host: encode a 4-D tensor map {W, H, P, Q} (row-major, dense) with box
// {bw, bh, 1, bq}: bq consecutive Q-slices of one P index per copy.
bool encode_map_4d(CUtensorMap* map, const void* base, int elem_bytes,
                   CUtensorMapDataType dtype, uint64_t W, uint64_t H, uint64_t P,
                   uint64_t Q, uint32_t bw, uint32_t bh, uint32_t bq,
                   const char** err);

}  // namespace nsc
