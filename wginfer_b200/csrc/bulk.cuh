// mbarrier and one-dimensional bulk-copy (cp.async.bulk, the copy engine
// without a tensor map) helpers. Every wait is bounded: a wait that runs out
// returns false and the caller records a device error instead of hanging.
#pragma once

#include "common.cuh"

namespace wgb {

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the copy engine.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// One arrival that also announces `bytes` of bulk copies completing on b.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// One plain arrival.
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// Waits for the phase of the given parity to complete; polls, and checks the
// SM cycle counter every 64 polls. false after max_cycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity, long long max_cycles) {
    long long t0 = 0;
    for (unsigned i = 0;; i++) {
        unsigned ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(smem_u32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 63) == 63) {
            const long long t = clock64();
            if (i == 63) t0 = t;
            else if (t - t0 > max_cycles) return false;
        }
    }
}
// 16-byte shared-memory load from a 32-bit shared address (an ld.shared, not
// a generic load the compiler must first resolve: measured 4.2 vs 5.4 cycles
// per step of a dependent FMA chain fed from dynamic shared memory).
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}

// Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global to shared memory; completion is counted on mbarrier b.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(b))
                 : "memory");
}

}  // namespace wgb
