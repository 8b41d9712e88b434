// Shared device helpers for the sm_100a decode-path kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "libm_expf.cuh"
#include "wginfer_b200.h"

namespace wgb {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs (queried at run time too)

// ---- element types -------------------------------------------------------
// Stores round to nearest even (bf16, f16). For finite values the bf16 result
// equals the reference's host conversion (utils/types.cpp:74-83).
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float load(float v) { return v; }
    static __device__ __forceinline__ float store(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
    // bf16 -> f32 is exact: the 16 bits become the high half of the f32
    // (an integer shift, kept off the conversion pipe)
    static __device__ __forceinline__ float load(__nv_bfloat16 v) {
        return __uint_as_float((uint32_t)__bfloat16_as_ushort(v) << 16);
    }
    static __device__ __forceinline__ __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float load(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half store(float v) { return __float2half_rn(v); }
};

template <typename T> __device__ __forceinline__ float ldf(const T *p, size_t i) {
    return Elem<T>::load(p[i]);
}
template <typename T> __device__ __forceinline__ void stf(T *p, size_t i, float v) {
    p[i] = Elem<T>::store(v);
}

// 16-byte vector of T.
template <typename T> struct Vec16 {
    static constexpr int N = 16 / sizeof(T);
    union {
        uint4 u;
        T e[N];
    };
};

__device__ __forceinline__ uint4 ld_global_nc_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
// Read-only load that allocates in L1 (operands every CTA of an SM re-reads).
__device__ __forceinline__ uint4 ld_global_l1_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
// Streaming load for data read exactly once (weights): evict-first in L2,
// expressed as an L2 cache-policy operand.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void *p, uint64_t pol) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(pol));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Single-precision sin, cos and pow evaluated in double precision and rounded
// once (correctly rounded with overwhelming probability). exp has its own
// restatement of the C library's algorithm (libm_expf.cuh), which matches the
// reference's std::exp(float) bit for bit.
__device__ __forceinline__ float sin_cr(float x) { return (float)sin((double)x); }
__device__ __forceinline__ float cos_cr(float x) { return (float)cos((double)x); }
__device__ __forceinline__ float pow_cr(float b, float e) { return (float)pow((double)b, (double)e); }

// rms_norm's 1 / sqrt(sum / n + eps), each operation rounded once
// (rms_norm_cpu.cpp:18-19: std::sqrt of a float is the correctly rounded sqrtf).
__device__ __forceinline__ float rms_scale(float sum, int n, float eps) {
    const float mean = __fdiv_rn(sum, (float)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch: let the next kernel in the stream launch now,
// and wait until the previous kernel's results are visible. Both are no-ops
// for a kernel launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Pulls [p, p + bytes) into L2, this CTA taking its 1/nctas share in
// 64 KB bulk prefetches (sizes and addresses kept 16-byte granular).
__device__ __forceinline__ void l2_prefetch_share(const void *p, size_t bytes, int cta, int nctas) {
    if (p == nullptr || bytes == 0) return;
    const size_t chunk = 64 * 1024;
    const size_t nchunks = (bytes + chunk - 1) / chunk;
    for (size_t c = (size_t)cta; c < nchunks; c += (size_t)nctas) {
        const size_t off = c * chunk;
        size_t n = bytes - off < chunk ? bytes - off : chunk;
        n &= ~(size_t)15;
        if (n)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((const char *)p + off), "r"((uint32_t)n)
                         : "memory");
    }
}

// Records the first bad value a kernel met ({code, value}) in the library's
// device error word (status.cu) instead of faulting.
__device__ __forceinline__ void record_device_error(unsigned long long *rec, int code, long long value) {
    if (rec != nullptr && atomicCAS(rec, 0ull, (unsigned long long)code) == 0ull)
        rec[1] = (unsigned long long)value;
}

}  // namespace wgb

// ---- host-side status plumbing (status.cpp) --------------------------------
namespace wgb {
int set_error(int status, const char *fmt, ...);
int check_launch(const char *what);
int current_numerics();
int sm_count();
unsigned long long *dev_error_ptr();
// Whether decode kernels are chained with programmatic dependent launch
// (default on; WGB_PDL=0 in the environment turns it off).
bool pdl_enabled();
}  // namespace wgb

#define WGB_REQUIRE(cond, status, ...)                    \
    do {                                                  \
        if (!(cond)) return ::wgb::set_error(status, __VA_ARGS__); \
    } while (0)

#define WGB_DISPATCH_FLOAT(dtype, T, ...)                                                    \
    switch (dtype) {                                                                         \
    case WGINFER_DTYPE_F32: { using T = float; __VA_ARGS__; break; }                         \
    case WGINFER_DTYPE_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }                \
    case WGINFER_DTYPE_F16: { using T = __half; __VA_ARGS__; break; }                        \
    default:                                                                                 \
        return ::wgb::set_error(WGB_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", (int)dtype); \
    }
