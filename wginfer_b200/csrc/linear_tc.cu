// Tensor-core GEMM for linear with more than 8 input rows (prefill, batched
// decode): out[M, N] = X[M, K] . W[N, K]^T on the 5th-generation tensor cores.
//
// A CTA owns 128 weight rows (the MMA's M dimension, one TMEM lane each) and
// TN input rows (the MMA's N dimension, TN in {16, 32, 64, 128, 256}); the
// f32 accumulator tile [128 x TN] lives in tensor memory. Warp 0 streams
// 64-wide K slices of W and X into a 4-stage shared-memory ring with TMA
// (cp.async.bulk.tensor, 128-byte swizzle, no multicast); one thread of
// warp 1 issues tcgen05.mma (kind::f16, bf16 in, f32 accumulate, 4 x K16 per
// slice) and frees each stage with tcgen05.commit; after the last slice all
// four warps read the accumulator with tcgen05.ld (warp w owns TMEM lanes
// 32w..32w+31, i.e. weight rows) and run the same epilogues as the GEMV path
// (decode_common.cuh): bias, residual, SwiGLU of adjacent gate/up rows, or
// RoPE + K/V append of adjacent rotation partners (the partner's value comes
// from the neighbouring lane by shuffle). Output writes are coalesced: for a
// fixed input row, the 32 lanes of a warp write 32 consecutive outputs.
// Roofline: tensor, 2*M*N*K flops.
//
// Every mbarrier wait is bounded; on a stall the kernel records an error in
// the device error word, skips the rest, waits (bounded) for copies in
// flight and always releases its tensor memory.
#include <cuda.h>

#include <atomic>

#include "common.cuh"
#include "decode_common.cuh"
#include "kernels.h"

namespace wgb {
namespace {

constexpr int kTcThreads = 128;
constexpr int kBK = 64;          // K elements per stage (128 bytes of bf16: one swizzle span)
constexpr int kTcMaxStages = 8;
constexpr int kTileW = 128;      // weight rows per CTA (MMA M)
constexpr long long kTcWaitCycles = 4000000000ll;  // a stage stalled this long (about 2 s) counts as a failure

__device__ __forceinline__ uint32_t s_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(uint64_t *b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(uint64_t *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(b)), "r"(bytes) : "memory");
}
// Bounded wait for the phase with the given parity: polls first, then
// checks the SM cycle counter (cheap, unlike %globaltimer) every 64 polls;
// false after kTcWaitCycles.
__device__ __forceinline__ bool mb_wait(uint64_t *b, unsigned parity) {
    long long t0 = 0;
    for (unsigned i = 0;; i++) {
        unsigned ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(s_u32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 63) == 63) {
            const long long t = clock64();
            if (i == 63) t0 = t;
            else if (t - t0 > kTcWaitCycles) return false;
        }
    }
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            s_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(s_u32(bar))
        : "memory");
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (start and stride in 16-byte units; version 1).
__device__ __forceinline__ uint64_t sw128_desc(const void *p) {
    const uint64_t addr = s_u32(p);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Instruction descriptor: bf16 A and B, f32 D, both K-major, M = 128, N = tn.
__host__ __device__ inline uint32_t idesc_bf16(int tn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(tn >> 3) << 17) | ((uint32_t)(kTileW >> 4) << 24);
}

// Stages in the ring: 4. Deeper rings for the narrow tiles were measured
// slower: their shared memory halves the CTAs resident per SM, and a CTA's
// throughput does not grow with its ring depth.
inline int tc_stages(int) { return 4; }
inline size_t tc_smem_bytes(int tn) {
    return 1024 + (size_t)tc_stages(tn) * ((size_t)kTileW * kBK * 2 + (size_t)tn * kBK * 2);
}
inline size_t tc_smem_max() {
    size_t m = 0;
    for (int tn = 16; tn <= 256; tn *= 2) m = tc_smem_bytes(tn) > m ? tc_smem_bytes(tn) : m;
    return m;
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, DecodeGemvParams p,
                   int tn, int nst) {
    using T = __nv_bfloat16;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[kTcMaxStages], empty[kTcMaxStages], done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_bad, s_issued;
    unsigned char *smem = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int a_bytes = kTileW * kBK * 2, b_bytes = tn * kBK * 2, st_bytes = a_bytes + b_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTileW, m0 = blockIdx.y * tn;
    const int ktiles = (p.K + kBK - 1) / kBK;
    const uint32_t ncols = tn <= 32 ? 32 : (uint32_t)tn;  // a power of two >= 32

    if (threadIdx.x == 0) {
        s_bad = 0;
        s_issued = 0;
        for (int i = 0; i < nst; i++) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], 1);
        }
        mb_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(&s_tmem)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;
    pdl_trigger();
    pdl_wait();  // X (and, for residuals, the output) come from the previous kernel

    if (warp == 0 && lane == 0) {
        // producer: TMA slices of W (128 rows) and X (tn rows) into the ring
        for (int kt = 0; kt < ktiles; kt++) {
            const int st = kt % nst;
            if (kt >= nst && !mb_wait(&empty[st], (unsigned)(((kt / nst) - 1) & 1))) {
                atomicExch(&s_bad, 1);
                break;
            }
            unsigned char *a = smem + (size_t)st * st_bytes;
            mb_expect_tx(&full[st], (unsigned)st_bytes);
            tma_load_2d(a, &tmW, kt * kBK, n0, &full[st]);
            tma_load_2d(a + a_bytes, &tmX, kt * kBK, m0, &full[st]);
            s_issued = kt + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        const uint32_t idesc = idesc_bf16(tn);
        for (int kt = 0; kt < ktiles; kt++) {
            const int st = kt % nst;
            if (!mb_wait(&full[st], (unsigned)((kt / nst) & 1))) {
                atomicExch(&s_bad, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const unsigned char *a = smem + (size_t)st * st_bytes;
#pragma unroll
            for (int k = 0; k < kBK / 16; k++)
                mma_bf16(tmem, sw128_desc(a + k * 32), sw128_desc(a + a_bytes + k * 32), idesc, (kt | k) != 0);
            mma_commit(&empty[st]);  // the stage is free once these MMAs have read it
        }
        mma_commit(&done);
    }
    __syncwarp();
    // epilogue: all four warps; warp w reads TMEM lanes 32w..32w+31 (weight rows)
    if (!mb_wait(&done, 0)) atomicExch(&s_bad, 1);
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const bool ok = !s_bad;
    if (ok) {
        const int n = n0 + warp * 32 + lane;
        for (int c0 = 0; c0 < tn; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const float v = __uint_as_float(r[j]);
                const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
                const int m = m0 + c0 + j;
                if ((lane & 1) == 0 && c0 + j < tn && m < p.M && n < p.N)
                    epilogue<T, EPI>(p, n >> 1, n, n + 1, n + 1 < p.N, m, v, partner);
            }
        }
    } else if (threadIdx.x == 0) {
        record_device_error(p.err, 6, blockIdx.x);
        // TMA copies may still be landing in the ring: wait (bounded) for
        // the last one issued into each stage before the CTA exits
        for (int kt = s_issued - 1; kt >= 0 && kt >= s_issued - nst; kt--)
            mb_wait(&full[kt % nst], (unsigned)((kt / nst) & 1));
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
}

// ---- host: tensor maps through the driver entry point (not linked) ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiledFn) nullptr;
        return (EncodeTiledFn)f;
    }();
    return fn;
}

// [rows, K] bf16 row-major, box [kBK, box_rows], 128-byte swizzle, zero fill.
bool make_map(CUtensorMap *tm, const void *base, int rows, int K, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Input rows per tile: the smallest power of two >= M up to 256 (the MMA's
// largest N; fewer re-reads of the weight tile), then halved (down to 16)
// while the grid would leave SMs idle; each halving re-reads the weights once
// more, mostly from L2.
int pick_tn(int M, int N) {
    int tn = 16;
    while (tn < M && tn < 256) tn *= 2;
    const long long wtiles = (N + kTileW - 1) / kTileW;
    while (tn > 16 && wtiles * ((M + tn - 1) / tn) < sm_count()) tn /= 2;
    return tn;
}

template <int EPI>
int launch_tc(const DecodeGemvParams &p, cudaStream_t s) {
    const int tn = pick_tn(p.M, p.N);
    CUtensorMap tmW, tmX;
    if (!make_map(&tmW, p.w, p.N, p.K, kTileW) || !make_map(&tmX, p.x, p.M, p.K, tn))
        return set_error(WGB_ERR_CUDA, "linear(tc): tensor map encoding failed");
    // the shared-memory limit is a per-device function attribute
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)tc_smem_max());
        if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "linear(tc): %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.N + kTileW - 1) / kTileW), (unsigned)((p.M + tn - 1) / tn));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = tc_smem_bytes(tn);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<EPI>, tmW, tmX, p, tn, tc_stages(tn));
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "linear(tc): %s", cudaGetErrorString(e));
    return WGB_OK;
}

}  // namespace

bool tc_gemm_ok(const DecodeGemvParams &p) {
    // TMA: 16-byte aligned bases and row strides; grid.y = M / tn <= 65535
    return p.M > 8 && p.K > 0 && p.K % 8 == 0 && aligned16(p.w) && aligned16(p.x) && p.N >= 1 && encode_fn() &&
           p.M <= 128 * 65535 && p.N < (1 << 30);
}

int tc_gemm(const DecodeGemvParams &p0, int epi, cudaStream_t s) {
    DecodeGemvParams p = p0;
    if (!p.err) p.err = dev_error_ptr();  // stalls are reported through the device error word
    if (epi == DG_EPI_SWIGLU) return launch_tc<EPI_SWIGLU>(p, s);
    if (epi == DG_EPI_ROPEKV) return launch_tc<EPI_ROPEKV>(p, s);
    return launch_tc<EPI_STORE>(p, s);
}

void tc_gemm_prepare() {
    const int lim = (int)tc_smem_max();
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_ROPEKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
}

bool linear_tc_supported(size_t M, size_t N, size_t K, const void *out, const void *x, const void *w) {
    DecodeGemvParams p{};
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.w = w;
    p.x = x;
    return M <= 128 * 65535 && N < (1u << 30) && K < (1u << 30) && tc_gemm_ok(p);
}

int linear_tc_bf16(void *out, const void *x, const void *w, const void *bias, const void *residual, int M, int N, int K,
                   cudaStream_t s) {
    DecodeGemvParams p{};
    p.w = w;
    p.x = x;
    p.M0 = p.M = M;
    p.N = N;
    p.K = K;
    p.groups = (N + 1) / 2;
    p.out = out;
    p.ldo = N;
    p.bias = bias;
    p.res = residual;
    p.err = dev_error_ptr();
    return tc_gemm(p, DG_EPI_STORE, s);
}

}  // namespace wgb
