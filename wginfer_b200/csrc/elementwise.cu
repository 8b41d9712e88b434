// add and swiglu: two-input, one-output streaming kernels.
//
// Each thread moves 16-byte vectors (8 bf16/f16 or 4 f32) with non-allocating
// loads, UNROLL vectors in flight before any store, over a grid sized to a
// whole number of waves of the SMs; the ragged tail (numel % vector) is done
// by scalar threads, so no access ever leaves the buffers (the reference's
// add read a full vector past the end when numel was not a multiple of it,
// src/ops/add/nvidia/add_nvidia.cu:7-43). Unaligned views (byte-offset
// slices) take a scalar grid-stride path. Roofline: HBM, 3 * numel * size
// bytes per call.
#include "common.cuh"

namespace wgb {
namespace {

struct AddOp {
    __device__ __forceinline__ float operator()(float a, float b) const { return __fadd_rn(a, b); }
};

// src/ops/swiglu/cpu/swiglu_cpu.cpp:11 evaluates up * gate / (1 + exp(-gate))
// with the product and the quotient each rounded once; REFERENCE keeps that
// literally, with the C library's expf restated (libm_expf.cuh). FAST uses the hardware exp2-based __expf
// and the approximate quotient __fdividef (a few ulp: relative error below
// 1e-6 for |gate| < 20, and 0 instead of a denormal once 1 + exp(-gate)
// passes 2^126): at bf16 the IEEE division and accurate expf made the op
// instruction-bound, well short of HBM bandwidth.
template <bool kRef> struct SwigluOp {
    __device__ __forceinline__ float operator()(float g, float u) const {
        if (kRef) return __fdiv_rn(__fmul_rn(u, g), __fadd_rn(1.0f, expf_glibc(-g)));
        return __fdividef(u * g, 1.0f + __expf(-g));
    }
};

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

template <typename T, class Op>
__global__ void __launch_bounds__(kThreads) ew2_vec_kernel(T *__restrict__ out, const T *__restrict__ a,
                                                           const T *__restrict__ b, size_t nvec, size_t n, Op op) {
    constexpr int V = Vec16<T>::N;
    const size_t stride = (size_t)gridDim.x * kThreads;
    // every pass requests all of its (up to kUnroll) vectors before the first
    // use; the last pass is predicated rather than finished one vector per
    // round trip
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < nvec; i += kUnroll * stride) {
        Vec16<T> va[kUnroll], vb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            if (i + u * stride < nvec) {
                va[u].u = ld_global_nc_v4(a + (i + u * stride) * V);
                vb[u].u = ld_global_nc_v4(b + (i + u * stride) * V);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            if (i + u * stride < nvec) {
                Vec16<T> vo;
#pragma unroll
                for (int e = 0; e < V; e++)
                    vo.e[e] = Elem<T>::store(op(Elem<T>::load(va[u].e[e]), Elem<T>::load(vb[u].e[e])));
                *reinterpret_cast<uint4 *>(out + (i + u * stride) * V) = vo.u;
            }
        }
    }
    // scalar tail
    if (blockIdx.x == 0) {
        for (size_t j = nvec * V + threadIdx.x; j < n; j += kThreads) stf(out, j, op(ldf(a, j), ldf(b, j)));
    }
}

template <typename T, class Op>
__global__ void __launch_bounds__(kThreads) ew2_scalar_kernel(T *out, const T *a, const T *b, size_t n, Op op) {
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (size_t)gridDim.x * kThreads)
        stf(out, i, op(ldf(a, i), ldf(b, i)));
}

template <typename T, class Op>
int launch_ew2(T *out, const T *a, const T *b, size_t n, cudaStream_t s, Op op, const char *name) {
    if (n == 0) return WGB_OK;
    constexpr int V = Vec16<T>::N;
    const int max_blocks = sm_count() * (2048 / kThreads);
    if (aligned16(out) && aligned16(a) && aligned16(b)) {
        // passes per thread: as few as a full grid allows; then the fewest
        // CTAs that cover the vectors in that many passes, so every thread
        // has (nearly) the same number of vectors. One pass: spread the
        // vectors over as many SMs as possible (one per thread).
        size_t nvec = n / V;
        const size_t per_pass = (size_t)kThreads * kUnroll;
        const size_t passes = (nvec + per_pass * max_blocks - 1) / (per_pass * max_blocks);
        size_t want = passes > 1 ? (nvec + per_pass * passes - 1) / (per_pass * passes) : (nvec + kThreads - 1) / kThreads;
        int blocks = (int)(want < 1 ? 1 : (want > (size_t)max_blocks ? max_blocks : want));
        ew2_vec_kernel<T, Op><<<blocks, kThreads, 0, s>>>(out, a, b, nvec, n, op);
    } else {
        size_t want = (n + kThreads - 1) / kThreads;
        int blocks = (int)(want > (size_t)max_blocks ? max_blocks : want);
        ew2_scalar_kernel<T, Op><<<blocks, kThreads, 0, s>>>(out, a, b, n, op);
    }
    return check_launch(name);
}

}  // namespace
}  // namespace wgb

extern "C" int wgb_add(void *c, const void *a, const void *b, wginferDataType_t dtype, size_t numel,
                       wginferStream_t stream) {
    WGB_REQUIRE(numel == 0 || (c && a && b), WGB_ERR_INVALID_ARGUMENT, "wgb_add: null pointer");
    WGB_DISPATCH_FLOAT(dtype, T,
        return wgb::launch_ew2((T *)c, (const T *)a, (const T *)b, numel, (cudaStream_t)stream, wgb::AddOp{}, "wgb_add"));
    return WGB_OK;
}

extern "C" int wgb_swiglu(void *out, const void *gate, const void *up, wginferDataType_t dtype, size_t numel,
                          wginferStream_t stream) {
    WGB_REQUIRE(numel == 0 || (out && gate && up), WGB_ERR_INVALID_ARGUMENT, "wgb_swiglu: null pointer");
    const bool ref = wgb::current_numerics() == WGB_NUMERICS_REFERENCE;
    if (ref) {
        WGB_DISPATCH_FLOAT(dtype, T,
            return wgb::launch_ew2((T *)out, (const T *)gate, (const T *)up, numel, (cudaStream_t)stream,
                                   wgb::SwigluOp<true>{}, "wgb_swiglu"));
    } else {
        WGB_DISPATCH_FLOAT(dtype, T,
            return wgb::launch_ew2((T *)out, (const T *)gate, (const T *)up, numel, (cudaStream_t)stream,
                                   wgb::SwigluOp<false>{}, "wgb_swiglu"));
    }
    return WGB_OK;
}
