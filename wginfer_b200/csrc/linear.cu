// linear: out[M, N] = in[M, K] . W[N, K]^T (+ bias), f32 accumulation.
//
// Dispatch (wgb_linear):
//  - FAST, bf16, M > kGemvMaxM, aligned: tcgen05 tensor-core GEMM
//    (linear_tc.cu) with the bias fused in its epilogue.
//  - FAST otherwise: the weight-streaming GEMV of decode_gemv.cu (a warp
//    owns two weight rows and a slice of K; lanes stream 16-byte weight
//    vectors evict-first and apply them to up to 8 input rows at once, so W
//    crosses HBM once per 8 rows; the bias is added before the single
//    rounding). Roofline: HBM, (N*K + M*K + M*N + N) * size bytes.
//  - REFERENCE: every output is one sequential f32 chain over k in order,
//    starting from 0 (+ bias), as src/ops/linear/cpu/linear_cpu.cpp:75-107
//    (f16/bf16) and :25-72 (f32) compute it; bf16/f16 products are exact in
//    f32, so an FMA there equals the reference's multiply-then-add, while f32
//    products are rounded before the add. Weight tiles stream through a
//    cp.async shared-memory ring so the chains never wait on HBM.
//  - Anything else (odd K, unaligned views): a scalar fallback.
#include <cuda_pipeline.h>

#include "common.cuh"
#include "kernels.h"

namespace wgb {
namespace {

constexpr int kGemvMaxM = 8;

// Output rounding: y = round(acc + bias); with a residual r (the model's
// fused skip connection) y = round(r + round(acc + bias)), i.e. exactly the
// reference's linear followed by its add (model.cpp:436-440, :459-463).
template <typename T>
__device__ __forceinline__ void store_out(T *out, const T *res, size_t idx, float s) {
    if (res) {
        const float r = Elem<T>::load(Elem<T>::store(s));
        s = __fadd_rn(ldf(res, idx), r);
    }
    stf(out, idx, s);
}

template <typename T>
__global__ void __launch_bounds__(256) gemv_scalar_kernel(T *out, const T *x, const T *w, const T *bias,
                                                          const T *res, int M, int N, int K) {
    const int warp = (blockIdx.x * 256 + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * 256) >> 5;
    for (int t = warp; t < M * N; t += nwarps) {
        const int m = t / N, n = t % N;
        float s = 0.f;
        for (int k = lane; k < K; k += 32) s = fmaf(ldf(x, (size_t)m * K + k), ldf(w, (size_t)n * K + k), s);
        s = warp_sum(s);
        if (lane == 0) {
            if (bias) s += ldf(bias, n);
            store_out(out, res, (size_t)m * N + n, s);
        }
    }
}

// ---- REFERENCE order ------------------------------------------------------
constexpr int kRefRows = 64;    // weight rows (threads) per CTA
constexpr int kRefStages = 4;   // cp.async ring depth
constexpr int kRefMT = 8;       // input rows per pass

template <bool kExactProduct>
__device__ __forceinline__ float chain_step(float acc, float xv, float wv) {
    // bf16/f16 products are exact in f32: fma == multiply-then-add
    return kExactProduct ? fmaf(xv, wv, acc) : __fadd_rn(acc, __fmul_rn(xv, wv));
}

template <typename T, int MT>
__global__ void __launch_bounds__(kRefRows) gemv_ref_kernel(T *out, const T *__restrict__ x,
                                                            const T *__restrict__ w, const T *__restrict__ bias,
                                                            const T *res, int M, int N, int K) {
    constexpr bool kExact = !std::is_same<T, float>::value;
    constexpr int V = 16 / sizeof(T);
    constexpr int KT = 128 / sizeof(T);   // k per tile: 64 (bf16/f16) or 32 (f32)
    constexpr int LDW = KT + V;           // padded row stride: 144 bytes, conflict-free 16-byte reads
    __shared__ __align__(16) T ws[kRefStages][kRefRows * LDW];
    __shared__ float xs[kRefStages][MT][KT];
    const int tid = threadIdx.x;
    const int n0 = blockIdx.x * kRefRows;
    const int n = n0 + tid;
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const int ntiles = (K + KT - 1) / KT;
    const bool vec = (K % V) == 0 && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);

    auto issue = [&](int t) {
        const int st = t % kRefStages;
        const int k0 = t * KT;
        const int kl = min(KT, K - k0);
        if (vec) {
            constexpr int vpr = KT / V;
            for (int c = tid; c < kRefRows * vpr; c += kRefRows) {
                const int r = c / vpr, cv = c % vpr;
                const int nn = n0 + r;
                if (nn < N && cv * V < kl)
                    __pipeline_memcpy_async(&ws[st][r * LDW + cv * V], w + (size_t)nn * K + k0 + cv * V, 16);
            }
        } else {
            for (int c = tid; c < kRefRows * KT; c += kRefRows) {
                const int r = c / KT, kk = c % KT;
                const int nn = n0 + r;
                if (nn < N && kk < kl) ws[st][r * LDW + kk] = w[(size_t)nn * K + k0 + kk];
            }
        }
        for (int c = tid; c < MT * KT; c += kRefRows) {
            const int m = c / KT, kk = c % KT;
            xs[st][m][kk] = (m < mt && kk < kl) ? ldf(x, (size_t)(m0 + m) * K + k0 + kk) : 0.f;
        }
        __pipeline_commit();
    };

    float acc[MT];
    const float b = (bias && n < N) ? ldf(bias, n) : 0.f;
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = __fadd_rn(0.f, b);

    for (int t = 0; t < kRefStages - 1; t++) {
        if (t < ntiles) issue(t);
        else __pipeline_commit();
    }
    for (int t = 0; t < ntiles; t++) {
        if (t + kRefStages - 1 < ntiles) issue(t + kRefStages - 1);
        else __pipeline_commit();
        __pipeline_wait_prior(kRefStages - 1);
        __syncthreads();
        const int st = t % kRefStages;
        const int kl = min(KT, K - t * KT);
        const T *wr = &ws[st][tid * LDW];
        if (kl == KT) {
#pragma unroll
            for (int k8 = 0; k8 < KT; k8 += V) {
                Vec16<T> wv;
                wv.u = *reinterpret_cast<const uint4 *>(wr + k8);
#pragma unroll
                for (int e = 0; e < V; e++) {
                    const float wf = Elem<T>::load(wv.e[e]);
#pragma unroll
                    for (int m = 0; m < MT; m++) acc[m] = chain_step<kExact>(acc[m], xs[st][m][k8 + e], wf);
                }
            }
        } else {
            for (int kk = 0; kk < kl; kk++) {
                const float wf = Elem<T>::load(wr[kk]);
#pragma unroll
                for (int m = 0; m < MT; m++) acc[m] = chain_step<kExact>(acc[m], xs[st][m][kk], wf);
            }
        }
        __syncthreads();
    }
    if (n < N) {
#pragma unroll
        for (int m = 0; m < MT; m++)
            if (m < mt) store_out(out, res, (size_t)(m0 + m) * N + n, acc[m]);
    }
}

template <typename T>
int launch_linear(T *out, const T *x, const T *w, const T *bias, const T *res, size_t M, size_t N, size_t K,
                  bool ref, cudaStream_t s) {
    constexpr int V = Vec16<T>::N;
    if (ref && M <= (size_t)kRefChainMaxM) {
        // a few rows: one chain per lane, weights streamed ahead (ref_decode.cu)
        DecodeGemvParams p{};
        p.w = w;
        p.x = x;
        p.M0 = (int)M;
        p.N = (int)N;
        p.K = (int)K;
        p.out = out;
        p.ldo = (int)N;
        p.bias = bias;
        p.res = res;
        p.err = dev_error_ptr();
        const wginferDataType_t dt = std::is_same<T, float>::value    ? WGINFER_DTYPE_F32
                                     : std::is_same<T, __half>::value ? WGINFER_DTYPE_F16
                                                                      : WGINFER_DTYPE_BF16;
        if (ref_chain_ok(dt, p)) {
            ref_decode_prepare();
            return ref_chain_gemv(dt, p, DG_PRO_PLAIN, DG_EPI_STORE, s);
        }
    }
    if (ref) {
        // one input row: one chain per thread; otherwise eight chains per thread
        const int mt = M == 1 ? 1 : kRefMT;
        dim3 grid((unsigned)((N + kRefRows - 1) / kRefRows), (unsigned)((M + mt - 1) / mt));
        WGB_REQUIRE(grid.y <= 65535, WGB_ERR_INVALID_ARGUMENT, "wgb_linear: M too large");
        if (mt == 1) gemv_ref_kernel<T, 1><<<grid, kRefRows, 0, s>>>(out, x, w, bias, res, (int)M, (int)N, (int)K);
        else gemv_ref_kernel<T, kRefMT><<<grid, kRefRows, 0, s>>>(out, x, w, bias, res, (int)M, (int)N, (int)K);
        return check_launch("linear(reference)");
    }
    const bool vec = (K % V) == 0 && aligned16(x) && aligned16(w);
    if (std::is_same<T, __nv_bfloat16>::value && vec && M > (size_t)kGemvMaxM && linear_tc_supported(M, N, K, out, x, w))
        return linear_tc_bf16(out, x, w, bias, res, (int)M, (int)N, (int)K, s);
    if (vec) {
        // the weight-streaming GEMV of decode_gemv.cu, plain prologue and store epilogue
        DecodeGemvParams p{};
        p.w = w;
        p.x = x;
        p.M0 = (int)M;
        p.N = (int)N;
        p.K = (int)K;
        p.groups = (int)((N + 1) / 2);
        p.out = out;
        p.ldo = (int)N;
        p.bias = bias;
        p.res = res;
        const wginferDataType_t dt = std::is_same<T, float>::value    ? WGINFER_DTYPE_F32
                                     : std::is_same<T, __half>::value ? WGINFER_DTYPE_F16
                                                                      : WGINFER_DTYPE_BF16;
        return decode_gemv(dt, p, DG_PRO_PLAIN, DG_EPI_STORE, s);
    }
    const size_t want = (M * N + 7) / 8;
    const int cap = sm_count() * 8;
    gemv_scalar_kernel<T><<<(int)(want < (size_t)cap ? want : cap), 256, 0, s>>>(out, x, w, bias, res, (int)M,
                                                                                (int)N, (int)K);
    return check_launch("linear(scalar)");
}

}  // namespace

int linear_forward(wginferDataType_t dtype, void *out, const void *x, const void *w, const void *bias,
                   const void *residual, int M, int N, int K, bool ref, cudaStream_t s) {
    WGB_DISPATCH_FLOAT(dtype, T,
        return launch_linear((T *)out, (const T *)x, (const T *)w, (const T *)bias, (const T *)residual, (size_t)M,
                             (size_t)N, (size_t)K, ref, s));
    return WGB_OK;
}

}  // namespace wgb

extern "C" int wgb_linear(void *out, const void *in, const void *weight, const void *bias, wginferDataType_t dtype,
                          size_t M, size_t N, size_t K, wginferStream_t stream) {
    if (M == 0 || N == 0) return WGB_OK;
    WGB_REQUIRE(out && in && weight, WGB_ERR_INVALID_ARGUMENT, "wgb_linear: null pointer");
    WGB_REQUIRE(M < (1u << 30) && N < (1u << 30) && K < (1u << 30), WGB_ERR_INVALID_ARGUMENT,
                "wgb_linear: size too large");
    const bool ref = wgb::current_numerics() == WGB_NUMERICS_REFERENCE;
    WGB_DISPATCH_FLOAT(dtype, T,
        return wgb::launch_linear((T *)out, (const T *)in, (const T *)weight, (const T *)bias, (const T *)nullptr, M,
                                  N, K, ref, (cudaStream_t)stream));
    return WGB_OK;
}
