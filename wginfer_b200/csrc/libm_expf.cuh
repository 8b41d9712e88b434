// Single-precision exp with the exact results of the GNU C library's expf.
//
// The reference's CPU ops call std::exp(float) (swiglu_cpu.cpp:11, the
// softmax of self_attention_cpu.cpp:72), i.e. glibc's expf. glibc's expf is
// not correctly rounded (it differs from the correctly rounded value on about
// 8e-5 of all floats), so REFERENCE numerics cannot use a correctly rounded
// exp and stay bit-identical. This is a restatement of glibc's published
// method (sysdeps/ieee754/flt-32/e_expf.c since glibc 2.27, from Arm's
// optimized-routines, Szabolcs Nagy 2017), written for both the host and the
// device:
//
//   k = round(x * 32/ln2), r = x * 32/ln2 - k       (r in [-1/2, 1/2])
//   exp(x) = 2^(k/32) * 2^(r/32)
//   2^(k/32): a 32-entry table of 2^(i/32) with the exponent k/32 added
//             to the bits
//   2^(r/32) ~ 1 + c2 r + c1 r^2 + c0 r^3          (in double)
//   result   = (float)(s * poly)                   (one rounding)
//
// The round-to-integer is the 1.5 * 2^52 shift trick. The x86-64 build of
// glibc that systems with FMA select (the __expf_fma variant) contracts the
// reduction into two fused multiply-adds; this restatement does the same, so
// it reproduces that variant on all 2^32 inputs. The test suite checks every
// input against the host C library. The table entries are the correctly
// rounded doubles of 2^(i/32) minus i << 47 (computed independently to 60
// digits); the polynomial is the published one of that implementation.
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define WGB_HD __host__ __device__ __forceinline__
#else
#include <cmath>
#define WGB_HD inline
#endif

namespace wgb {

#define WGB_EXP2_32_TABLE                                                                                \
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,       \
        0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,   \
        0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,   \
        0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,   \
        0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,   \
        0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,   \
        0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,   \
        0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull

#if defined(__CUDACC__)
// device copy (global memory, cached in L1); host code uses the array below
__device__ const uint64_t kExp2Tab32Dev[32] = {WGB_EXP2_32_TABLE};
#endif
static const uint64_t kExp2Tab32Host[32] = {WGB_EXP2_32_TABLE};

namespace libm_detail {
WGB_HD double as_double(uint64_t u) {
    double d;
    memcpy(&d, &u, 8);
    return d;
}
WGB_HD uint64_t as_u64(double d) {
    uint64_t u;
    memcpy(&u, &d, 8);
    return u;
}
WGB_HD uint32_t as_u32(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
WGB_HD float as_float(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
WGB_HD double dfma(double a, double b, double c) {
#if defined(__CUDA_ARCH__)
    return __fma_rn(a, b, c);
#else
    return std::fma(a, b, c);
#endif
}
WGB_HD double dmul(double a, double b) {
#if defined(__CUDA_ARCH__)
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}
WGB_HD double dsub(double a, double b) {
#if defined(__CUDA_ARCH__)
    return __dsub_rn(a, b);
#else
    return a - b;
#endif
}
}  // namespace libm_detail

// expf exactly as the GNU C library computes it (errno aside).
WGB_HD float expf_glibc(float x) {
    using namespace libm_detail;
    constexpr double kInvLn2x32 = 0x1.71547652b82fep+0 * 32.0;
    constexpr double kShift = 0x1.8p+52;
    constexpr double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    constexpr double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    constexpr double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const uint32_t ux = as_u32(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {  // |x| >= 88, inf or nan
        if (ux == 0xff800000u) return 0.0f;          // -inf
        if (abstop >= 0x7f8u) return x + x;          // +inf, nan
        if (x > 0x1.62e42ep6f) return as_float(0x7f800000u);  // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;         // underflow
    }
    const double xd = (double)x;
    double kd = dfma(kInvLn2x32, xd, kShift);  // k in the low bits of the mantissa
    const uint64_t ki = as_u64(kd);
    kd = dsub(kd, kShift);
    const double r = dfma(kInvLn2x32, xd, -kd);
#if defined(__CUDA_ARCH__)
    uint64_t t = kExp2Tab32Dev[ki & 31];
#else
    uint64_t t = kExp2Tab32Host[ki & 31];
#endif
    t += ki << 47;
    const double s = as_double(t);
    const double z = dfma(c0, r, c1);
    const double r2 = dmul(r, r);
    double y = dfma(c2, r, 1.0);
    y = dfma(z, r2, y);
    return (float)dmul(y, s);
}

#undef WGB_EXP2_32_TABLE

}  // namespace wgb
