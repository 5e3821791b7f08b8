// pipeline.cuh -- shared-memory pipelines fed by the bulk-copy (TMA) engine:
// mbarrier set-up, arrival, bounded waits, 1-D cp.async.bulk copies and 2-D
// and 3-D tensor-map box copies from global to shared memory.  Every copy has one
// destination, this CTA's shared memory, and reads this GPU's own memory.
//
// Every wait is bounded.  When a wait gives up it sets the sticky error word
// (the library's device status, read by clq_device_status) and returns false;
// a wait also returns false at once when the word is already set, so one
// expired wait makes every other waiter fall through instead of stalling.
#pragma once

#include <cstdint>

namespace clq {
namespace pipe {

constexpr uint32_t kWaitLimit = 1u << 26;  // polls before a wait gives up (seconds, with the back-off)

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes initialised barriers visible to the bulk-copy engine.
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with PARITY; false (and *err set) when it gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_test(bar, parity)) return true;
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_test(bar, parity)) return true;
        if (*(volatile int*)err) return false;
        if (i > 64) __nanosleep(32);
    }
    atomicExch(err, CLQ_ERR_TIMEOUT);
    return false;
}
// Bounded wait that ignores the error word: before a CTA exits, so that the
// copies it issued have landed.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); i++) {
        if (mbar_test(bar, parity)) return;
        if (i > 64) __nanosleep(64);
    }
}
// BYTES (a multiple of 16) from global SRC to shared DST, both 16-byte
// aligned; completion is counted on BAR's transaction count.
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// The box of the 2-D tensor map MAP (a kernel parameter) at (X, Y) -- X the
// innermost coordinate, in elements, with X times the element size a multiple
// of 16 bytes -- to shared DST (128-byte aligned); completion is counted on
// BAR's transaction count (the full box, out-of-range elements zero-filled).
__device__ __forceinline__ void tensor_copy_2d(void* dst, const void* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// An L2 policy that marks lines read once (a weight stream) first for
// eviction, so that they do not push out small, reused data.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// tensor_copy_2d with the L2 cache POLICY.
__device__ __forceinline__ void tensor_copy_2d_hint(void* dst, const void* map, int x, int y, uint64_t* bar,
                                                    uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// The same for a 3-D map (coordinates innermost first).
__device__ __forceinline__ void tensor_copy_3d_hint(void* dst, const void* map, int x, int y, int z, uint64_t* bar,
                                                    uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// Programmatic dependent launch: wait until the grids this one depends on
// have completed and their writes are visible (a no-op without the launch
// attribute), and let the next grid in the stream start its prologue.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
// Named barrier over the first THREADS threads of the CTA (ID 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace pipe
}  // namespace clq
