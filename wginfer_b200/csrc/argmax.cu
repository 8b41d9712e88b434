// argmax over each row of vals[rows, numel]: the first index of the maximum
// under '>' in f32 (src/ops/argmax/cpu/argmax_cpu.cpp:26-47), bit-exact.
//
// A thread-block cluster of up to 8 CTAs shares one row (fewer when there are
// many rows, so that all CTAs fit in one wave): each CTA reduces
// its slice with 16-byte loads to one 64-bit key per CTA, and CTA 0 of the
// cluster folds the keys of the others through distributed shared memory,
// so no global scratch and no second launch are needed. Per 16-byte vector a
// thread does a branch-free max tree and one compare with its running
// maximum, remembering the first vector that set it; the element index is
// found once, at the end, by re-reading that vector. (An element-wise
// compare-and-select chain made the op instruction-bound at bf16.) Key = (order-
// preserving bits of the value) << 32 | (0xFFFFFFFF - index): the largest
// key is the largest value at the smallest index. -0 is folded into +0
// (they compare equal under '>'); NaN never wins unless it is element 0,
// where the sequential scan keeps it, as the reference does.
// Roofline: HBM, rows*numel*size + rows*(8+size) bytes.
#include <cooperative_groups.h>

#include <atomic>

#include "argmax_key.cuh"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace wgb {
namespace {

constexpr int kCluster = 8;
// threads per CTA: 512 (two CTAs per SM) when the rows fill the GPU, 256
// for a few rows
constexpr int kThreadsWide = 512, kThreadsFew = 256;
// 16-byte vectors in flight per thread: 8 when the rows fill the GPU; 10 for
// a few rows, where a 151936-wide bf16 row on 8 CTAs is then one round trip
// (latency, not bandwidth, is what a few rows pay for)
constexpr int kBWide = 8, kBFew = 10;

// Per-thread running best over the thread's elements, which it visits in
// increasing index order: strict '>' keeps the first index of a tie, and NaN
// never compares greater. The 64-bit key is formed only when threads merge.
struct Best {
    float v;
    uint32_t i;  // 0xFFFFFFFF: nothing seen yet
};
template <typename T>
__device__ __forceinline__ void consider(Best &b, T x, uint32_t idx) {
    const float v = Elem<T>::load(x);
    if (v > b.v || (b.i == 0xFFFFFFFFu && !isnan(v))) {
        b.v = v;
        b.i = idx;
    }
}
// Maximum of a 16-byte vector by a max tree (NaN operands lose to numbers;
// a vector of NaN only gives NaN).
template <typename T> __device__ __forceinline__ float vec_max(const Vec16<T> &r);
template <> __device__ __forceinline__ float vec_max<__nv_bfloat16>(const Vec16<__nv_bfloat16> &r) {
    const __nv_bfloat162 *p = reinterpret_cast<const __nv_bfloat162 *>(&r.u);
    const __nv_bfloat162 m = __hmax2(__hmax2(p[0], p[1]), __hmax2(p[2], p[3]));
    return Elem<__nv_bfloat16>::load(__hmax(__low2bfloat16(m), __high2bfloat16(m)));
}
template <> __device__ __forceinline__ float vec_max<__half>(const Vec16<__half> &r) {
    const __half2 *p = reinterpret_cast<const __half2 *>(&r.u);
    const __half2 m = __hmax2(__hmax2(p[0], p[1]), __hmax2(p[2], p[3]));
    return __half2float(__hmax(__low2half(m), __high2half(m)));
}
template <> __device__ __forceinline__ float vec_max<float>(const Vec16<float> &r) {
    return fmaxf(fmaxf(r.e[0], r.e[1]), fmaxf(r.e[2], r.e[3]));
}

template <typename T, bool kVec, int kB, int kThreads>
__global__ void __launch_bounds__(kThreads, 2) argmax_cluster_kernel(int64_t *max_idx, T *max_val, const T *vals,
                                                                  size_t numel, int64_t *lens, int64_t maxlen) {
    constexpr int V = Vec16<T>::N;
    __shared__ unsigned long long red[kThreads / 32];
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank(), ns = cluster.num_blocks();
    const size_t row = blockIdx.x / ns;
    const T *x = vals + row * numel;
    // launched with programmatic dependent launch: this CTA may start while
    // the kernel that writes `vals` finishes; it waits for it before reading
    pdl_trigger();
    pdl_wait();
    Best bt{-INFINITY, 0xFFFFFFFFu};

    if (kVec) {
        const size_t nvec = numel / V;
        const size_t per = (nvec + ns - 1) / ns;
        const size_t v0 = rank * per < nvec ? rank * per : nvec, v1 = v0 + per < nvec ? v0 + per : nvec;
        // batches of kB vectors per thread, the last batch predicated, so a
        // thread's slice costs ceil(slice / kB) round trips; per vector one
        // compare: the first vector (in index order) holding the thread's
        // maximum is remembered
        float best = -INFINITY;
        long long bvec = -1;
        for (size_t i = v0 + threadIdx.x; i < v1; i += kB * kThreads) {
            Vec16<T> r[kB];
#pragma unroll
            for (int u = 0; u < kB; u++)
                if (i + u * kThreads < v1) r[u].u = ld_global_nc_v4(x + (i + u * kThreads) * V);
#pragma unroll
            for (int u = 0; u < kB; u++) {
                if (i + u * kThreads < v1) {
                    const float m = vec_max<T>(r[u]);
                    if (m > best || (bvec < 0 && m == m)) {
                        best = m;
                        bvec = (long long)(i + u * kThreads);
                    }
                }
            }
        }
        if (bvec >= 0) {  // the first element of that vector equal to the maximum
            Vec16<T> r;
            r.u = ld_global_nc_v4(x + (size_t)bvec * V);
#pragma unroll
            for (int e = V - 1; e >= 0; e--)
                if (Elem<T>::load(r.e[e]) == best) bt.i = (uint32_t)(bvec * V + e);
            bt.v = best;
        }
    } else {
        const size_t per = (numel + ns - 1) / ns;
        const size_t e0 = rank * per < numel ? rank * per : numel, e1 = e0 + per < numel ? e0 + per : numel;
        for (size_t i = e0 + threadIdx.x; i < e1; i += kThreads) consider(bt, x[i], (uint32_t)i);
    }
    unsigned long long best = bt.i == 0xFFFFFFFFu ? 0ull : make_key(bt.v, bt.i);  // 0: below every real key
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
        for (unsigned r = 1; r < ns; r++) {
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
        // decode step: the row's sequence has grown by the token just chosen
        if (lens && lens[row] < maxlen) lens[row] += 1;
    }
    cluster.sync();  // keep peers' shared memory alive until CTA 0 has read it
}

template <typename T>
int launch_argmax(int64_t *idx, T *val, const T *vals, size_t rows, size_t numel, cudaStream_t s,
                  int64_t *lens = nullptr, int64_t maxlen = 0) {
    constexpr int V = Vec16<T>::N;
    const bool vec = aligned16(vals) && (numel % V) == 0;
    // CTAs per row: up to kCluster, but no more than one wave of resident
    // CTAs over all rows (the resident count comes from the occupancy query,
    // cached per device and variant)
    static std::atomic<int> resident[64][2];
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = dev >= 0 && dev < 64 ? resident[dev][vec ? 1 : 0].load(std::memory_order_relaxed) : 0;
    if (per_sm <= 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &per_sm,
                vec ? argmax_cluster_kernel<T, true, kBWide, kThreadsWide>
                    : argmax_cluster_kernel<T, false, kBWide, kThreadsWide>,
                kThreadsWide, 0) != cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
        if (dev >= 0 && dev < 64) resident[dev][vec ? 1 : 0].store(per_sm, std::memory_order_relaxed);
    }
    // few rows (every row gets the full cluster): the deeper batch
    const bool few = rows * kCluster <= (size_t)sm_count();
    const size_t wave = (size_t)sm_count() * per_sm;
    size_t ns = rows >= wave ? 1 : wave / rows;
    if (ns > (size_t)kCluster) ns = kCluster;
    if (ns < 1) ns = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * ns));
    cfg.blockDim = dim3(vec && few ? kThreadsFew : kThreadsWide);
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)ns;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e;
    if (vec && few)
        e = cudaLaunchKernelEx(&cfg, argmax_cluster_kernel<T, true, kBFew, kThreadsFew>, idx, val, vals, numel, lens, maxlen);
    else if (vec)
        e = cudaLaunchKernelEx(&cfg, argmax_cluster_kernel<T, true, kBWide, kThreadsWide>, idx, val, vals, numel, lens, maxlen);
    else e = cudaLaunchKernelEx(&cfg, argmax_cluster_kernel<T, false, kBWide, kThreadsWide>, idx, val, vals, numel, lens, maxlen);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "wgb_argmax: %s", cudaGetErrorString(e));
    return check_launch("wgb_argmax");
}

}  // namespace
}  // namespace wgb

namespace wgb {
// Greedy step of batched decode: argmax of each logit row into tokens[row],
// and lens[row] += 1 (up to maxlen) once the row's token is chosen, in one
// launch.
int argmax_rows_advance(int64_t *tokens, const void *logits, wginferDataType_t dtype, size_t rows, size_t numel,
                        int64_t *lens, int64_t maxlen, cudaStream_t s) {
    WGB_DISPATCH_FLOAT(dtype, T,
        return launch_argmax(tokens, (T *)nullptr, (const T *)logits, rows, numel, s, lens, maxlen));
    return WGB_OK;
}
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
