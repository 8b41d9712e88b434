// The 64-bit argmax key shared by the argmax kernels and the fused
// lm_head + argmax epilogues: (order-preserving bits of the value) << 32 |
// (0xFFFFFFFF - index), so the largest key is the largest value at the
// smallest index, the tie rule of the reference's sequential scan
// (src/ops/argmax/cpu/argmax_cpu.cpp:26-47: strict '>', first index kept).
// -0 is folded into +0 (they compare equal under '>'). NaN never wins: its
// key is 0, below every real key; the scan keeps a NaN only at index 0,
// which the finalising step checks separately.
#pragma once

#include "common.cuh"

namespace wgb {

__device__ __forceinline__ unsigned long long make_key(float v, uint32_t idx) {
    if (v == 0.f) v = 0.f;  // -0 -> +0
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

__device__ __forceinline__ unsigned long long key_or_zero(float v, uint32_t idx) {
    return isnan(v) ? 0ull : make_key(v, idx);
}

__device__ __forceinline__ unsigned long long warp_max_key(unsigned long long k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
    }
    return k;
}

// Index of the argmax from the merged key of a row whose element 0 is x0.
__device__ __forceinline__ int64_t key_index(unsigned long long key, float x0) {
    if (isnan(x0) || key == 0ull) return 0;
    return (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

}  // namespace wgb
