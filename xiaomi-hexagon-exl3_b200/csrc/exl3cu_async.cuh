// Asynchronous-copy and barrier primitives for sm_100a: shared-memory
// mbarriers, bulk (TMA, non-tensor) global->shared copies, programmatic
// dependent launch, and a device status word for bounded waits.
//
// Every wait here is bounded.  A wait that runs out of iterations returns
// false; the caller records kStatusWaitTimeout in its translation unit's
// device status word, skips the remaining compute but still passes every
// barrier, so a stuck copy can never hang the GPU.  The host reads and clears
// the word with exl3cu_device_status().
#pragma once
#include <stdint.h>

namespace exl3cu {

constexpr unsigned kStatusWaitTimeout = 1u;
constexpr unsigned kStatusBadIndex = 2u;   // an index argument read on the device was out of range
constexpr unsigned kWaitSpins = 1u << 22;  // try_wait rounds before giving up (each may suspend briefly)

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// Wait for the phase with the given parity to complete; false after kWaitSpins rounds.
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    const uint32_t addr = smem_addr(bar);
    for (unsigned i = 0; i < kWaitSpins; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Same, but a thread whose phase is not complete sleeps (up to about a
// microsecond per round, woken early when the phase completes) instead of
// spinning, so that waiting warps leave their issue slots to the warps that
// share the scheduler.  Bounded: false after kSleepWaitRounds rounds (about a
// second).
constexpr unsigned kSleepWaitRounds = 1u << 20;

__device__ __forceinline__ bool mbar_wait_sleep(uint64_t * bar, uint32_t parity) {
    const uint32_t addr = smem_addr(bar);
    for (unsigned i = 0; i < kSleepWaitRounds; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity), "r"(1000u)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) into this
// CTA's shared memory, completing transaction bytes on `bar`.  No multicast.
__device__ __forceinline__ void bulk_g2s(void * dst_smem, const void * src_gmem, uint32_t bytes, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// L2 policy for data read once per pass (streamed weights): evicted first, so
// that it does not push the activations and outputs of a chain of kernels out
// of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// bulk_g2s with an L2 cache policy (l2_evict_first_policy for streamed weights).
__device__ __forceinline__ void bulk_g2s_hint(void * dst_smem, const void * src_gmem, uint32_t bytes, uint64_t * bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_addr(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Peer-exchange words: (epoch << 32 | float bits).  Four values go out as two 16-byte stores
// whose 8-byte elements are each single-copy atomic at system scope, so a reader on any GPU sees
// a value together with the epoch it was stored under.  `p` is 16-byte aligned.
__device__ __forceinline__ void store_pairs4(unsigned long long * p, float4 v, unsigned epoch) {
    const unsigned long long e = (unsigned long long)epoch << 32;
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(e | __float_as_uint(v.x)),
                 "l"(e | __float_as_uint(v.y))
                 : "memory");
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p + 2), "l"(e | __float_as_uint(v.z)),
                 "l"(e | __float_as_uint(v.w))
                 : "memory");
}

__device__ __forceinline__ unsigned long long load_pair(const unsigned long long * p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_primary() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace exl3cu
