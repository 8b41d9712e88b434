// argmax over each row of vals[rows, numel]: the first index of the maximum
// under '>' in f32 (src/ops/argmax/cpu/argmax_cpu.cpp:26-47), bit-exact.
//
// A thread-block cluster of kCluster CTAs shares one row: each CTA reduces
// its slice with 16-byte loads to one 64-bit key per CTA, and CTA 0 of the
// cluster folds the keys of the others through distributed shared memory,
// so no global scratch and no second launch are needed. Key = (order-
// preserving bits of the value) << 32 | (0xFFFFFFFF - index): the largest
// key is the largest value at the smallest index. -0 is folded into +0
// (they compare equal under '>'); NaN never wins unless it is element 0,
// where the sequential scan keeps it, as the reference does.
// Roofline: HBM, rows*numel*size + rows*(8+size) bytes.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace wgb {
namespace {

constexpr int kCluster = 8;
constexpr int kThreads = 512;

__device__ __forceinline__ unsigned long long make_key(float v, uint32_t idx) {
    if (v == 0.f) v = 0.f;  // -0 -> +0
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

template <typename T>
__device__ __forceinline__ void consider(unsigned long long &best, T x, uint32_t idx) {
    float v = Elem<T>::load(x);
    if (!isnan(v)) {
        unsigned long long k = make_key(v, idx);
        best = k > best ? k : best;
    }
}

template <typename T, bool kVec>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    argmax_cluster_kernel(int64_t *max_idx, T *max_val, const T *vals, size_t numel) {
    constexpr int V = Vec16<T>::N;
    __shared__ unsigned long long red[kThreads / 32];
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank();
    const size_t row = blockIdx.x / kCluster;
    const T *x = vals + row * numel;
    unsigned long long best = 0ull;  // below every real key

    if (kVec) {
        const size_t nvec = numel / V;
        const size_t per = (nvec + kCluster - 1) / kCluster;
        const size_t v0 = rank * per, v1 = v0 + per < nvec ? v0 + per : nvec;
        size_t i = v0 + threadIdx.x;
        for (; i + 3 * kThreads < v1; i += 4 * kThreads) {
            Vec16<T> r[4];
#pragma unroll
            for (int u = 0; u < 4; u++) r[u].u = ld_global_nc_v4(x + (i + u * kThreads) * V);
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int e = 0; e < V; e++) consider(best, r[u].e[e], (uint32_t)((i + u * kThreads) * V + e));
        }
        for (; i < v1; i += kThreads) {
            Vec16<T> r;
            r.u = ld_global_nc_v4(x + i * V);
#pragma unroll
            for (int e = 0; e < V; e++) consider(best, r.e[e], (uint32_t)(i * V + e));
        }
    } else {
        const size_t per = (numel + kCluster - 1) / kCluster;
        const size_t e0 = rank * per, e1 = e0 + per < numel ? e0 + per : numel;
        for (size_t i = e0 + threadIdx.x; i < e1; i += kThreads) consider(best, x[i], (uint32_t)i);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        unsigned long long b = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
            b = other > b ? other : b;
        }
        if (threadIdx.x == 0) red[0] = b;
    }
    cluster.sync();  // every CTA's red[0] is final and visible cluster-wide
    if (rank == 0 && threadIdx.x == 0) {
        unsigned long long b = red[0];
        for (unsigned r = 1; r < kCluster; r++) {
            unsigned long long o = *cluster.map_shared_rank(&red[0], r);
            b = o > b ? o : b;
        }
        int64_t idx;
        if (numel == 0) {
            max_idx[row] = 0;
            if (max_val) max_val[row] = Elem<T>::store(0.f);
        } else {
            if (isnan(Elem<T>::load(x[0])) || b == 0ull) idx = 0;
            else idx = (int64_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
            max_idx[row] = idx;
            if (max_val) max_val[row] = x[idx];
        }
    }
    cluster.sync();  // keep peers' shared memory alive until CTA 0 has read it
}

template <typename T>
int launch_argmax(int64_t *idx, T *val, const T *vals, size_t rows, size_t numel, cudaStream_t s) {
    constexpr int V = Vec16<T>::N;
    const bool vec = aligned16(vals) && (numel % V) == 0;
    dim3 grid((unsigned)(rows * kCluster));
    if (vec) argmax_cluster_kernel<T, true><<<grid, kThreads, 0, s>>>(idx, val, vals, numel);
    else argmax_cluster_kernel<T, false><<<grid, kThreads, 0, s>>>(idx, val, vals, numel);
    return check_launch("wgb_argmax");
}

}  // namespace
}  // namespace wgb

extern "C" int wgb_argmax_rows(int64_t *max_idx, void *max_val, const void *vals, wginferDataType_t dtype,
                               size_t rows, size_t numel, wginferStream_t stream) {
    if (rows == 0) return WGB_OK;
    WGB_REQUIRE(max_idx && (vals || numel == 0), WGB_ERR_INVALID_ARGUMENT, "wgb_argmax: null pointer");
    WGB_REQUIRE(numel < 0xFFFFFFFFull, WGB_ERR_INVALID_ARGUMENT, "wgb_argmax: numel must be < 2^32 - 1");
    WGB_REQUIRE(rows <= (1u << 26), WGB_ERR_INVALID_ARGUMENT, "wgb_argmax: too many rows");
    WGB_DISPATCH_FLOAT(dtype, T,
        return wgb::launch_argmax(max_idx, (T *)max_val, (const T *)vals, rows, numel, (cudaStream_t)stream));
    return WGB_OK;
}

extern "C" int wgb_argmax(int64_t *max_idx, void *max_val, const void *vals, wginferDataType_t dtype, size_t numel,
                          wginferStream_t stream) {
    WGB_REQUIRE(max_val != nullptr, WGB_ERR_INVALID_ARGUMENT, "wgb_argmax: null max_val");
    return wgb_argmax_rows(max_idx, max_val, vals, dtype, 1, numel, stream);
}
