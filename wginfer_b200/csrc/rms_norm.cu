// rms_norm: y = x * w * (mean(x^2) + eps)^-1/2 per row.
//
// FAST: the row is read from HBM once into registers with 16-byte loads (a
// warp per row up to 256 vectors, a 256-thread CTA per row up to 2048
// vectors), squares are summed in f32 with warp shuffles, and the scaled
// row is written from the same registers. Other sizes or unaligned views use
// a two-pass CTA-per-row kernel (second read hits L2).
// REFERENCE: the sum of squares is one sequential f32 chain per row in index
// order (src/ops/rms_norm/cpu/rms_norm_cpu.cpp:11-17), done by one thread
// over the row staged in shared memory.
// Both modes form mean = sum / N, scale = 1 / sqrt(mean + eps) and
// y = (x * w) * scale with IEEE round-to-nearest at each step, as the
// reference does (rms_norm_cpu.cpp:18-26). Roofline: HBM, (2*M*N + N)*size B.
#include "common.cuh"

namespace wgb {
namespace {

template <typename T, int VPL>
__global__ void __launch_bounds__(256) rms_warp_kernel(T *__restrict__ out, const T *__restrict__ in,
                                                       const T *__restrict__ w, int M, int N, float eps) {
    constexpr int V = Vec16<T>::N;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    // launched with programmatic dependent launch: wait for the kernel that
    // writes `in` before reading it (and before writing `out`)
    pdl_trigger();
    pdl_wait();
    if (row >= M) return;
    const int nvec = N / V;
    const T *x = in + (size_t)row * N;
    Vec16<T> r[VPL], wr[VPL];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < VPL; u++) {  // x and the norm weight in one round trip
        int vi = lane + u * 32;
        if (vi < nvec) {
            r[u].u = ld_global_nc_v4(x + (size_t)vi * V);
            wr[u].u = ld_global_l1_v4(w + (size_t)vi * V);  // every row reads w: keep it in L1
        }
    }
#pragma unroll
    for (int u = 0; u < VPL; u++) {
        int vi = lane + u * 32;
        if (vi < nvec) {
#pragma unroll
            for (int e = 0; e < V; e++) {
                float f = Elem<T>::load(r[u].e[e]);
                ss = fmaf(f, f, ss);
            }
        }
    }
    ss = warp_sum(ss);
    const float sc = rms_scale(ss, N, eps);
    T *y = out + (size_t)row * N;
#pragma unroll
    for (int u = 0; u < VPL; u++) {
        int vi = lane + u * 32;
        if (vi < nvec) {
            Vec16<T> o;
#pragma unroll
            for (int e = 0; e < V; e++)
                o.e[e] = Elem<T>::store(__fmul_rn(__fmul_rn(Elem<T>::load(r[u].e[e]), Elem<T>::load(wr[u].e[e])), sc));
            *reinterpret_cast<uint4 *>(y + (size_t)vi * V) = o.u;
        }
    }
}

template <typename T, int VPT, int NT>
__global__ void __launch_bounds__(NT) rms_block_kernel(T *__restrict__ out, const T *__restrict__ in,
                                                       const T *__restrict__ w, int M, int N, float eps) {
    constexpr int V = Vec16<T>::N;
    __shared__ float red[NT / 32];
    const int row = blockIdx.x;
    const int nvec = N / V;
    const T *x = in + (size_t)row * N;
    Vec16<T> r[VPT], wr[VPT];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < VPT; u++) {  // x and the norm weight in one round trip
        int vi = threadIdx.x + u * NT;
        if (vi < nvec) {
            r[u].u = ld_global_nc_v4(x + (size_t)vi * V);
            wr[u].u = ld_global_l1_v4(w + (size_t)vi * V);  // every row reads w: keep it in L1
        }
    }
#pragma unroll
    for (int u = 0; u < VPT; u++) {
        int vi = threadIdx.x + u * NT;
        if (vi < nvec) {
#pragma unroll
            for (int e = 0; e < V; e++) {
                float f = Elem<T>::load(r[u].e[e]);
                ss = fmaf(f, f, ss);
            }
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = (threadIdx.x & 31) < NT / 32 ? red[threadIdx.x & 31] : 0.f;
    tot = warp_sum(tot);
    const float sc = rms_scale(tot, N, eps);
    T *y = out + (size_t)row * N;
#pragma unroll
    for (int u = 0; u < VPT; u++) {
        int vi = threadIdx.x + u * NT;
        if (vi < nvec) {
            Vec16<T> o;
#pragma unroll
            for (int e = 0; e < V; e++)
                o.e[e] = Elem<T>::store(__fmul_rn(__fmul_rn(Elem<T>::load(r[u].e[e]), Elem<T>::load(wr[u].e[e])), sc));
            *reinterpret_cast<uint4 *>(y + (size_t)vi * V) = o.u;
        }
    }
}

// Any N / alignment: two passes per row, CTA per row (grid-stride over rows).
template <typename T>
__global__ void __launch_bounds__(256) rms_generic_kernel(T *out, const T *in, const T *w, int M, int N, float eps) {
    __shared__ float red[8];
    for (int row = blockIdx.x; row < M; row += gridDim.x) {
        const T *x = in + (size_t)row * N;
        float ss = 0.f;
        for (int i = threadIdx.x; i < N; i += 256) {
            float f = ldf(x, i);
            ss = fmaf(f, f, ss);
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = (threadIdx.x & 31) < 8 ? red[threadIdx.x & 31] : 0.f;
        tot = warp_sum(tot);
        const float sc = rms_scale(tot, N, eps);
        T *y = out + (size_t)row * N;
        for (int i = threadIdx.x; i < N; i += 256) stf(y, i, __fmul_rn(__fmul_rn(ldf(x, i), ldf(w, i)), sc));
        __syncthreads();
    }
}

// REFERENCE order. The row is staged as f32 in shared memory (dynamic, up to
// kRefSmemFloats) so the single summing thread reads at shared-memory latency;
// longer rows are summed straight from global memory.
constexpr int kRefSmemFloats = 12288;
template <typename T>
__global__ void __launch_bounds__(256) rms_ref_kernel(T *out, const T *in, const T *w, int M, int N, float eps) {
    extern __shared__ float rowbuf[];
    __shared__ float s_scale;
    const bool staged = N <= kRefSmemFloats;
    for (int row = blockIdx.x; row < M; row += gridDim.x) {
        const T *x = in + (size_t)row * N;
        if (staged)
            for (int i = threadIdx.x; i < N; i += 256) rowbuf[i] = ldf(x, i);
        __syncthreads();
        if (threadIdx.x == 0) {
            float sum = 0.f;
            if (staged) {
                for (int i = 0; i < N; i++) sum = __fadd_rn(sum, __fmul_rn(rowbuf[i], rowbuf[i]));
            } else {
                for (int i = 0; i < N; i++) {
                    float f = ldf(x, i);
                    sum = __fadd_rn(sum, __fmul_rn(f, f));
                }
            }
            s_scale = rms_scale(sum, N, eps);
        }
        __syncthreads();
        const float sc = s_scale;
        T *y = out + (size_t)row * N;
        for (int i = threadIdx.x; i < N; i += 256) stf(y, i, __fmul_rn(__fmul_rn(ldf(x, i), ldf(w, i)), sc));
        __syncthreads();
    }
}

template <typename T>
int launch_rms(T *out, const T *in, const T *w, size_t M, size_t N, float eps, cudaStream_t s) {
    constexpr int V = Vec16<T>::N;
    const int grid_cap = sm_count() * 16;
    if (current_numerics() == WGB_NUMERICS_REFERENCE) {
        size_t smem = N <= (size_t)kRefSmemFloats ? N * sizeof(float) : 0;
        int blocks = (int)(M < (size_t)grid_cap ? M : grid_cap);
        rms_ref_kernel<T><<<blocks, 256, smem, s>>>(out, in, w, (int)M, (int)N, eps);
        return check_launch("wgb_rms_norm");
    }
    const bool vec_ok = (N % V) == 0 && aligned16(out) && aligned16(in) && aligned16(w);
    const size_t nvec = N / V;
    if (vec_ok && nvec <= 32 * 8) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((M + 7) / 8));
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = pdl_enabled() ? 1 : 0;
        cudaError_t e;
        if (nvec <= 32 * 2) e = cudaLaunchKernelEx(&cfg, rms_warp_kernel<T, 2>, out, in, w, (int)M, (int)N, eps);
        else if (nvec <= 32 * 4) e = cudaLaunchKernelEx(&cfg, rms_warp_kernel<T, 4>, out, in, w, (int)M, (int)N, eps);
        else if (nvec <= 32 * 6) e = cudaLaunchKernelEx(&cfg, rms_warp_kernel<T, 6>, out, in, w, (int)M, (int)N, eps);
        else e = cudaLaunchKernelEx(&cfg, rms_warp_kernel<T, 8>, out, in, w, (int)M, (int)N, eps);
        if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "wgb_rms_norm: %s", cudaGetErrorString(e));
    } else if (vec_ok && nvec <= 256 * 8) {
        // up to 4 vectors of the row (and 4 of the weight) per thread: the
        // longest rows take 512 threads rather than 8 vectors a thread,
        // which halved the CTAs resident per SM
        if (nvec <= 256 * 2) rms_block_kernel<T, 2, 256><<<(int)M, 256, 0, s>>>(out, in, w, (int)M, (int)N, eps);
        else if (nvec <= 256 * 4) rms_block_kernel<T, 4, 256><<<(int)M, 256, 0, s>>>(out, in, w, (int)M, (int)N, eps);
        else rms_block_kernel<T, 4, 512><<<(int)M, 512, 0, s>>>(out, in, w, (int)M, (int)N, eps);
    } else {
        int blocks = (int)(M < (size_t)grid_cap ? M : grid_cap);
        rms_generic_kernel<T><<<blocks, 256, 0, s>>>(out, in, w, (int)M, (int)N, eps);
    }
    return check_launch("wgb_rms_norm");
}

}  // namespace
}  // namespace wgb

extern "C" int wgb_rms_norm(void *out, const void *in, const void *weight, wginferDataType_t dtype, size_t M,
                            size_t N, float eps, wginferStream_t stream) {
    if (M == 0 || N == 0) return WGB_OK;
    WGB_REQUIRE(out && in && weight, WGB_ERR_INVALID_ARGUMENT, "wgb_rms_norm: null pointer");
    WGB_REQUIRE(M < (1u << 31) && N < (1u << 31), WGB_ERR_INVALID_ARGUMENT, "wgb_rms_norm: size too large");
    WGB_DISPATCH_FLOAT(dtype, T,
        return wgb::launch_rms((T *)out, (const T *)in, (const T *)weight, M, N, eps, (cudaStream_t)stream));
    return WGB_OK;
}
