// REFERENCE-numerics decode kernels for a few input rows (decode at batch
// <= 4): the token-identical path, made fast.
//
// The reference CPU backend sums every dot product as ONE sequential f32
// chain in index order (linear_cpu.cpp:86-99, rms_norm_cpu.cpp:11-17,
// self_attention_cpu.cpp:37-89), so a token-identical decode step is bounded
// below by its longest chains: K dependent adds per output (4 cycles each on
// the FMA pipe), i.e. ~3.1 us for K = 1536 and ~18.2 us for K = 8960, plus
// two L-long chains in attention. These kernels keep every chain at that
// rate and hide everything else behind it:
//
// ref_chain_kernel — one projection (linear) with every output one chain:
//   lane = weight row (32 rows per warp), MT input rows per lane (MT
//   independent chains). Each warp streams its rows' weights through its own
//   shared-memory ring: a stage is 32 rows x 128 bytes, and a ring slot is
//   one TMA box of J consecutive stages (cp.async.bulk.tensor over a 3-D
//   view of the matrix, 128-byte swizzle so the lanes' 16-byte reads of 32
//   different rows are bank-conflict free; completion counted on an
//   mbarrier per slot), issued a whole ring ahead of the chains, and before
//   the kernel waits for its predecessor (programmatic dependent launch):
//   weights do not depend on it. Measured on B200, a warp's boxes complete
//   about one every 0.35 us whatever their size, so the box size sets the
//   bandwidth: 4 KB boxes held a warp to ~12 GB/s; 32 KB boxes stream the
//   down projection at 1.9 TB/s over 48 warps and 16 KB boxes the lm_head at
//   6.5 TB/s. (Ragged K takes one-stage 2-D boxes.) bf16/f16 products are exact in f32, so an FMA equals the
//   reference's multiply-then-add; f32 products are rounded first. The bias
//   starts the chain (sum = 0; sum += bias), as the reference does.
//   Warps are independent after the prologue; a CTA of NW warps shares one
//   copy of the input rows, and a persistent grid walks the row blocks.
//   Prologue RMS: each CTA computes the rms_norm of its input rows itself, in
//   the reference's order (one chain over the row, then x * w * scale with
//   both products rounded), while its first weight stages arrive.
//   Epilogues (decode_common.cuh): STORE (+ residual), SWIGLU of adjacent
//   gate/up rows with the C library's expf restated (libm_expf.cuh), ROPEKV
//   of adjacent rotation partners (+ the K/V cache append), and ARGMAX: the
//   lm_head logits are stored and folded into one 64-bit (value, index) key
//   per input row; the CTA that finishes last writes the greedy token and
//   advances the sequence length, so the decode step needs no argmax launch.
//   Roofline: the chains (K x 4 cycles) for the narrow projections; HBM
//   (N K size bytes) for gate/up and lm_head.
//
// ref_attn_decode_kernel — one query row (the newest token of a sequence)
//   against its cached keys, per (sequence, head), on a cluster of 8 CTAs:
//   scores (a d-long chain per key) split over the cluster and written to
//   every CTA through distributed shared memory (one cluster barrier); every
//   CTA takes the max, exp, the L-long sequential sum and the division
//   itself (the same operations in the same order as its peers), then runs
//   16 of the 128 output columns' L-long chains of round(p * v) over its V
//   column slice, copied into shared memory while the scores were computed.
#include <cooperative_groups.h>
#include <cuda_pipeline.h>

#include <atomic>
#include <cfloat>

#include "argmax_key.cuh"
#include "bulk.cuh"
#include "common.cuh"
#include "decode_common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace wgb {
namespace {

constexpr int kRcLanes = 32;        // weight rows per warp (one chain owner per lane)
constexpr int kRcStageBytes = 128;  // bytes of one weight row per stage
constexpr int kRcStage = kRcLanes * kRcStageBytes;  // one stage of a warp: 4 KB
constexpr int kRcMaxSlots = 16;     // ring slots per warp, at most
constexpr int kRcMaxWarps = 4;
constexpr int kRcBarBytes = 1024;   // mbarriers at the start of shared memory (then 1 KB alignment slack)
constexpr long long kRcWaitCycles = 4000000000ll;  // a stage stalled this long (about 2 s) is a failure
constexpr int kRcErrCode = 8;       // device error code of a stalled stage
// dynamic shared memory per CTA: the 227 KB of an SM less room for the
// kernels' static shared variables
constexpr size_t kSmemLimit = 226 * 1024;

template <typename T> struct RcGeom {
    static constexpr int V = 16 / sizeof(T);
    static constexpr int KT = kRcStageBytes / sizeof(T);  // K elements per stage
};

// barriers (+ alignment slack), the rings (nw x ns slots of J stages), the
// input rows [mt][K] and the norm weight [K], both in the element type
size_t rc_smem_bytes(int nw, int ns, int J, int mt, int K, size_t es) {
    return 2 * kRcBarBytes + (size_t)nw * ns * J * kRcStage + (size_t)(mt + 1) * K * es;
}

template <bool kExact>
__device__ __forceinline__ float chain_step(float acc, float x, float w) {
    return kExact ? fmaf(x, w, acc) : __fadd_rn(acc, __fmul_rn(x, w));
}

// V chain steps acc = round(acc + x[e] * w[e]), e = 0..V-1 in order, over
// two 16-byte vectors of T. bf16 and f16 use the mixed-precision FMA (16-bit
// operands, f32 accumulator, one rounding): their products are exact in
// f32, so it equals the reference's multiply-then-add and needs no
// unpacking instructions. f32 rounds the product first, as the reference.
template <typename T> __device__ __forceinline__ void chain_vec(float &acc, const uint4 &x, const uint4 &w);
template <> __device__ __forceinline__ void chain_vec<__nv_bfloat16>(float &acc, const uint4 &x, const uint4 &w) {
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; q++)
        asm volatile("{\n .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %1;\n mov.b32 {wl, wh}, %2;\n"
            " fma.rn.f32.bf16 %0, xl, wl, %0;\n fma.rn.f32.bf16 %0, xh, wh, %0;\n}"
            : "+f"(acc)
            : "r"(xs[q]), "r"(ws[q]));
}
template <> __device__ __forceinline__ void chain_vec<__half>(float &acc, const uint4 &x, const uint4 &w) {
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; q++)
        asm volatile("{\n .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %1;\n mov.b32 {wl, wh}, %2;\n"
            " fma.rn.f32.f16 %0, xl, wl, %0;\n fma.rn.f32.f16 %0, xh, wh, %0;\n}"
            : "+f"(acc)
            : "r"(xs[q]), "r"(ws[q]));
}
template <> __device__ __forceinline__ void chain_vec<float>(float &acc, const uint4 &x, const uint4 &w) {
    acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(x.x), __uint_as_float(w.x)));
    acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(x.y), __uint_as_float(w.y)));
    acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(x.z), __uint_as_float(w.z)));
    acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(x.w), __uint_as_float(w.w)));
}

template <typename T> __device__ __forceinline__ float round_t(float v) { return Elem<T>::load(Elem<T>::store(v)); }

// Coherent (L2) load of one element written by another CTA of this launch.
template <typename T> __device__ __forceinline__ float ld_cg(const T *p) {
    if constexpr (sizeof(T) == 4) {
        return __ldcg(reinterpret_cast<const float *>(p));
    } else {
        const unsigned short u = __ldcg(reinterpret_cast<const unsigned short *>(p));
        T v;
        memcpy(&v, &u, 2);
        return Elem<T>::load(v);
    }
}

// Copies n elements (n * sizeof(T) a multiple of 16, both ends 16-byte
// aligned) into shared memory with every thread's 16-byte cp.async issued
// at once; committed as one group.
template <typename T> __device__ __forceinline__ void stage_copy(T *dst, const T *src, int n) {
    constexpr int V = 16 / sizeof(T);
    for (int i = threadIdx.x; i < n / V; i += blockDim.x) __pipeline_memcpy_async(dst + i * V, src + i * V, 16);
    __pipeline_commit();
}

template <int MT> struct ChainAcc {
    float v[MT];
};

// One full stage (128 bytes of each row) of chain steps: the stage's 16-byte
// operands are all loaded first, then its steps run (loads and steps are
// volatile asm, so the compiler keeps that order). wr: this lane's weight row
// in the ring (16-byte chunk c at c ^ sw); xr: input row 0 at this stage;
// xrow: bytes between input rows.
template <typename T, int MT>
__device__ __forceinline__ ChainAcc<MT> chain_stage(ChainAcc<MT> acc, uint32_t wr, uint32_t xr, int sw, uint32_t xrow) {
    constexpr int VPS = kRcStageBytes / 16;
    uint4 wv[VPS], xv[MT][VPS];
#pragma unroll
    for (int v = 0; v < VPS; v++) {
        wv[v] = lds128(wr + (uint32_t)((v ^ sw) << 4));
#pragma unroll
        for (int m = 0; m < MT; m++) xv[m][v] = lds128(xr + m * xrow + (uint32_t)(v * 16));
    }
#pragma unroll
    for (int v = 0; v < VPS; v++)
#pragma unroll
        for (int m = 0; m < MT; m++) chain_vec<T>(acc.v[m], xv[m][v], wv[v]);
    return acc;
}

// tmW: tma_map_row_stages view of the weights with J-stage boxes (J > 1), or
// the tma_map_rows view with one-stage boxes (J == 1); ns ring slots per warp.
// J is a template parameter so that a box's stages are one unrolled block of
// straight-line code (a runtime-bounded stage loop cost 1.3 cycles per chain
// step).
template <typename T, int MT, int PRO, int EPI, int J>
__global__ void __launch_bounds__(32 * kRcMaxWarps)
    ref_chain_kernel(const __grid_constant__ CUtensorMap tmW, DecodeGemvParams p, int ns) {
    constexpr int V = 16 / sizeof(T), KT = kRcStageBytes / sizeof(T);
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ float s_scale[MT];
    const int nw = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = p.K, N = p.N, M = p.M;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem) + warp * ns;
    // rings start on the first 1 KB boundary after the barriers (128-byte swizzle)
    const uint32_t sbase = smem_u32(smem);
    unsigned char *rings = smem + (((sbase + kRcBarBytes + 1023u) & ~1023u) - sbase);
    const int slot_bytes = J * kRcStage;
    unsigned char *ring = rings + (size_t)warp * ns * slot_bytes;
    T *xs = reinterpret_cast<T *>(rings + (size_t)nw * ns * slot_bytes);  // [MT][K] input rows
    T *nws = xs + (size_t)MT * K;                                          // [K] norm weight (RMS)

    const int nst = (K + KT - 1) / KT;  // stages per row block
    const int nbox = (nst + J - 1) / J;  // boxes (ring tiles) per row block
    const int nblocks = (N + kRcLanes - 1) / kRcLanes;
    // this warp's row blocks: first, first + step, ...
    const int first = blockIdx.x * nw + warp, step = gridDim.x * nw;
    const int myblocks = first < nblocks ? (nblocks - 1 - first) / step + 1 : 0;
    const int ntiles = myblocks * nbox;

    if (lane == 0) {
        for (int i = 0; i < ns; i++) mbar_init(&bar[i], 1);
        mbar_init_fence();
    }
    __syncwarp();
    // tile t = (row block first + (t / nbox) * step, stages J (t % nbox) ...) -> slot t % ns;
    // a box is always counted whole (rows past N and stages past K arrive as zeros)
    auto issue = [&](int t) {
        if (lane == 0) {
            uint64_t *b = &bar[t % ns];
            unsigned char *dst = ring + (size_t)(t % ns) * slot_bytes;
            const int r0 = (first + (t / nbox) * step) * kRcLanes;
            mbar_arrive_expect_tx(b, (unsigned)slot_bytes);
            if (J > 1) tma_load_box3(dst, &tmW, 0, r0, (t % nbox) * J, b);
            else tma_load_box(dst, &tmW, (t % nbox) * KT, r0, b);
        }
    };
    int issued = 0;
    for (; issued < ntiles && issued < ns; issued++) issue(issued);
    // operands that do not depend on the previous kernel: the norm weight
    if (PRO == DG_PRO_RMS) stage_copy(nws, reinterpret_cast<const T *>(p.norm_w), K);

    // let the next kernel launch and start its own weight copies
    pdl_trigger();
    pdl_wait();

    // input rows -> shared memory (rows >= M zero), one round trip
    stage_copy(xs, reinterpret_cast<const T *>(p.x), M * K);
    for (int i = M * K / V + threadIdx.x; i < MT * K / V; i += blockDim.x)
        reinterpret_cast<uint4 *>(xs)[i] = make_uint4(0u, 0u, 0u, 0u);
    // the residuals of this warp's first row block, requested now (STORE)
    float resv[MT];
    {
        const int row = first * kRcLanes + lane;
#pragma unroll
        for (int m = 0; m < MT; m++)
            resv[m] = (EPI == DG_EPI_STORE && p.res && m < M && first < nblocks && row < N)
                          ? ldf(reinterpret_cast<const T *>(p.res), (size_t)m * p.ldo + row)
                          : 0.f;
    }
    __pipeline_wait_prior(0);
    __syncthreads();
    if (PRO == DG_PRO_RMS) {
        // rms_norm_cpu.cpp:11-19: sum += v * v in index order, then
        // 1 / sqrt(sum / N + eps); one lane per input row
        if (threadIdx.x < M) {
            const uint32_t xr = smem_u32(xs + (size_t)threadIdx.x * K);
            float sum = 0.f;
            int v = 0;
            for (; v + 4 <= K / V; v += 4) {  // four vectors loaded, then their chain steps
                uint4 q[4];
#pragma unroll
                for (int u = 0; u < 4; u++) q[u] = lds128(xr + (uint32_t)((v + u) * 16));
#pragma unroll
                for (int u = 0; u < 4; u++) chain_vec<T>(sum, q[u], q[u]);
            }
            for (; v < K / V; v++) {
                const uint4 q = lds128(xr + (uint32_t)(v * 16));
                chain_vec<T>(sum, q, q);
            }
            s_scale[threadIdx.x] = rms_scale(sum, K, p.eps);
        }
        __syncthreads();
        // rms_norm_cpu.cpp:22-26: round(v * w * scale), rounded after each
        // product, then to the element type
        for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
            const int m = i / K, k = i - m * K;
            xs[i] = Elem<T>::store(__fmul_rn(__fmul_rn(Elem<T>::load(xs[i]), Elem<T>::load(nws[k])), s_scale[m]));
        }
        __syncthreads();
    }

    const T *bias = reinterpret_cast<const T *>(p.bias);
    const uint32_t ring_s = smem_u32(ring), xs_s = smem_u32(xs);
    int t = 0;
    bool failed = false;
    for (int bi = 0; bi < myblocks && !failed; bi++) {
        const int row = (first + bi * step) * kRcLanes + lane;
        const bool live = row < N;
        const float b0 = (bias && live) ? ldf(bias, row) : 0.f;
        ChainAcc<MT> acc;
#pragma unroll
        for (int m = 0; m < MT; m++) acc.v[m] = __fadd_rn(0.f, b0);
        // boxes of J whole stages (no per-stage test in this loop: a branch
        // there cost 2 of the 8 cycles per chain step), then a box of fewer
        // stages, then the ragged stage (one-stage boxes only)
        const int full_st = K / KT;
        const int nfull = full_st / J;
        const uint32_t xrow = (uint32_t)(K * (int)sizeof(T));
        for (int bx = 0; bx < nfull; bx++, t++) {
            const int slot = t % ns;
            const bool ok = mbar_wait(&bar[slot], (unsigned)((t / ns) & 1), kRcWaitCycles);
            if (__any_sync(0xffffffffu, !ok)) {
                failed = true;
                break;
            }
            const uint32_t wbox = ring_s + (uint32_t)(slot * slot_bytes + lane * kRcStageBytes);
            const uint32_t xbox = xs_s + (uint32_t)(bx * J * KT * (int)sizeof(T));
#pragma unroll
            for (int j = 0; j < J; j++)
                acc = chain_stage<T, MT>(acc, wbox + (uint32_t)(j * kRcStage),
                                         xbox + (uint32_t)(j * KT * (int)sizeof(T)), lane & 7, xrow);
            __syncwarp();  // every lane is done with this slot before it is refilled
            if (issued < ntiles) issue(issued++);
        }
        if (!failed && nfull * J < full_st) {
            const int slot = t % ns;
            const bool ok = mbar_wait(&bar[slot], (unsigned)((t / ns) & 1), kRcWaitCycles);
            if (__any_sync(0xffffffffu, !ok)) {
                failed = true;
            } else {
                const uint32_t wbox = ring_s + (uint32_t)(slot * slot_bytes + lane * kRcStageBytes);
                for (int s = nfull * J; s < full_st; s++)
                    acc = chain_stage<T, MT>(acc, wbox + (uint32_t)((s - nfull * J) * kRcStage),
                                             xs_s + (uint32_t)(s * KT * (int)sizeof(T)), lane & 7, xrow);
                __syncwarp();
                if (issued < ntiles) issue(issued++);
                t++;
            }
        }
        if (!failed && full_st < nst) {
            // the ragged last stage (K not a whole number of stages: one-stage boxes)
            const int slot = t % ns;
            const bool ok = mbar_wait(&bar[slot], (unsigned)((t / ns) & 1), kRcWaitCycles);
            if (__any_sync(0xffffffffu, !ok)) {
                failed = true;
            } else {
                const uint32_t wr = ring_s + (uint32_t)(slot * slot_bytes + lane * kRcStageBytes);
                const uint32_t xr = xs_s + (uint32_t)(full_st * KT * (int)sizeof(T));
                const int nv = (K - full_st * KT) / V;
                for (int v = 0; v < nv; v++) {
                    const uint4 wv = lds128(wr + (uint32_t)((v ^ (lane & 7)) << 4));
#pragma unroll
                    for (int m = 0; m < MT; m++)
                        chain_vec<T>(acc.v[m], lds128(xr + (uint32_t)((m * K + v * V) * (int)sizeof(T))), wv);
                }
                __syncwarp();
                if (issued < ntiles) issue(issued++);
                t++;
            }
        }
        if (failed) break;
        // epilogue of this row block
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m >= M) break;
            const float a = acc.v[m];
            if (EPI == DG_EPI_STORE) {
                if (live) {
                    const size_t i = (size_t)m * p.ldo + row;
                    float v = a;
                    if (p.res) v = __fadd_rn(bi == 0 ? resv[m] : ldf(reinterpret_cast<const T *>(p.res), i), round_t<T>(a));
                    stf(reinterpret_cast<T *>(p.out), i, v);
                }
            } else if (EPI == DG_EPI_SWIGLU) {
                // rows 2j, 2j + 1 are gate j and up j (swiglu_cpu.cpp:11)
                const float other = __shfl_xor_sync(0xffffffffu, a, 1);
                if (live && (lane & 1) == 0) {
                    const float gg = round_t<T>(a), uu = round_t<T>(other);
                    stf(reinterpret_cast<T *>(p.out), (size_t)m * p.ldo + row / 2,
                        __fdiv_rn(__fmul_rn(uu, gg), __fadd_rn(1.0f, expf_glibc(-gg))));
                }
            } else if (EPI == DG_EPI_ROPEKV) {
                // rows 2g, 2g + 1: rotation partners of a q/k head, or two v values
                const float other = __shfl_xor_sync(0xffffffffu, a, 1);
                if (live && (lane & 1) == 0) {
                    const int g = row / 2;
                    const int64_t pos = p.pos[m];
                    const int half = p.dh >> 1;
                    float2 cs = make_float2(0.f, 0.f);
                    if (g < (p.nh + p.nkvh) * half && pos >= 0 && pos < p.maxseq)
                        cs = p.table[(size_t)pos * half + (g % half)];
                    rope_kv_store<T>(p, g, row + 1 < N, m, a, other, pos, cs);
                }
            } else {  // DG_EPI_ARGMAX
                if (live) stf(reinterpret_cast<T *>(p.out), (size_t)m * p.ldo + row, a);
                unsigned long long key = live ? key_or_zero(round_t<T>(a), (uint32_t)row) : 0ull;
                key = warp_max_key(key);
                if (lane == 0 && key != 0ull) {
                    atomicMax(&p.amax_keys[m], key);
                    __threadfence();
                }
            }
        }
    }
    if (failed) {
        if (lane == 0) record_device_error(p.err, kRcErrCode, (long long)first);
        // let the copies still in flight land before the shared memory goes away
        for (int u = t; u < issued; u++) mbar_wait(&bar[u % ns], (unsigned)((u / ns) & 1), kRcWaitCycles / 16);
    }
    if (EPI == DG_EPI_ARGMAX) {
        // the CTA that finishes last turns the keys into tokens
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned done = atomicAdd(p.amax_count, 1u);
            if (done == gridDim.x - 1) {
                __threadfence();
                for (int m = 0; m < M; m++) {
                    const unsigned long long key = atomicExch(&p.amax_keys[m], 0ull);
                    const float x0 = ld_cg(reinterpret_cast<const T *>(p.out) + (size_t)m * p.ldo);
                    p.tokens[m] = key_index(key, x0);
                    if (p.lens && p.lens[m] < p.maxlen) p.lens[m] += 1;
                }
                atomicExch(p.amax_count, 0u);
            }
        }
    }
}

// (Launch shapes are chosen so that the CTAs of a launch are resident
// together: one CTA per SM at most, see rc_plan.)

template <typename T, int MT, int PRO, int EPI> void rc_set_attr() {
    // the launch reports what is wrong if an attribute is refused
    if (cudaFuncSetAttribute(ref_chain_kernel<T, MT, PRO, EPI, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit) != cudaSuccess)
        cudaGetLastError();
    if (cudaFuncSetAttribute(ref_chain_kernel<T, MT, PRO, EPI, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit) != cudaSuccess)
        cudaGetLastError();
    if (cudaFuncSetAttribute(ref_chain_kernel<T, MT, PRO, EPI, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit) != cudaSuccess)
        cudaGetLastError();
}

// Launch plan: warps per CTA (one for narrow projections, so more SMs pull
// weights; four when there are many row blocks, sharing one copy of the
// input rows), stages per box J (8 for one warp, 4 for four; 1 when K is
// not a whole number of stages or is shorter than a box; J is one of 1, 4,
// 8, the compiled variants) and ring slots per warp (up to 5, as many as
// one CTA per SM leaves room for, at least 2). The grid never exceeds one
// CTA per SM: every CTA is resident at once, and extra row blocks are
// walked by the persistent loop.
struct RcPlan {
    int nw, ns, J;
    size_t smem;
};
RcPlan rc_plan(int N, int K, int mt, size_t es) {
    const int nblocks = (N + kRcLanes - 1) / kRcLanes;
    const int KT = kRcStageBytes / (int)es;
    const int nst = (K + KT - 1) / KT;
    RcPlan pl;
    pl.nw = nblocks >= 2 * sm_count() ? kRcMaxWarps : 1;
    for (;;) {
        pl.J = K % KT ? 1 : (pl.nw == 1 ? 8 : 4);
        if (pl.J > nst) pl.J = nst >= 4 ? 4 : 1;
        const int want = pl.J == 1 ? kRcMaxSlots : 5;
        for (pl.ns = want; pl.ns > 2 && rc_smem_bytes(pl.nw, pl.ns, pl.J, mt, K, es) > kSmemLimit; pl.ns--) {
        }
        if (rc_smem_bytes(pl.nw, pl.ns, pl.J, mt, K, es) <= kSmemLimit || pl.nw == 1) break;
        pl.nw--;
    }
    while (pl.J > 1 && rc_smem_bytes(pl.nw, pl.ns, pl.J, mt, K, es) > kSmemLimit) pl.J = pl.J == 8 ? 4 : 1;
    pl.smem = rc_smem_bytes(pl.nw, pl.ns, pl.J, mt, K, es);
    return pl;
}

template <typename T, int MT, int PRO, int EPI> int launch_rc(const DecodeGemvParams &p0, cudaStream_t s) {
    DecodeGemvParams p = p0;
    p.M = p.M0;
    const RcPlan pl = rc_plan(p.N, p.K, MT, sizeof(T));
    CUtensorMap tm;
    const bool mapped = pl.J > 1 ? tma_map_row_stages(&tm, p.w, (int)sizeof(T), p.N, p.K, kRcLanes, pl.J)
                                 : tma_map_rows(&tm, p.w, (int)sizeof(T), p.N, p.K, kRcLanes);
    if (!mapped) return set_error(WGB_ERR_CUDA, "ref_chain_gemv: tensor map for [%d, %d] refused", p.N, p.K);
    const int nblocks = (p.N + kRcLanes - 1) / kRcLanes;
    const int ctas = (nblocks + pl.nw - 1) / pl.nw;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(ctas < sm_count() ? ctas : sm_count()));
    cfg.blockDim = dim3((unsigned)(32 * pl.nw));
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e;
    if (pl.J == 8) e = cudaLaunchKernelEx(&cfg, ref_chain_kernel<T, MT, PRO, EPI, 8>, tm, p, pl.ns);
    else if (pl.J == 4) e = cudaLaunchKernelEx(&cfg, ref_chain_kernel<T, MT, PRO, EPI, 4>, tm, p, pl.ns);
    else e = cudaLaunchKernelEx(&cfg, ref_chain_kernel<T, MT, PRO, EPI, 1>, tm, p, pl.ns);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "ref_chain_gemv: %s", cudaGetErrorString(e));
    return check_launch("ref_chain_gemv");
}

template <typename T, int PRO, int EPI> int launch_rc_m(const DecodeGemvParams &p, cudaStream_t s) {
    if (p.M0 <= 1) return launch_rc<T, 1, PRO, EPI>(p, s);
    if (p.M0 <= 2) return launch_rc<T, 2, PRO, EPI>(p, s);
    return launch_rc<T, 4, PRO, EPI>(p, s);
}

template <typename T> int launch_rc_t(const DecodeGemvParams &p, int pro, int epi, cudaStream_t s) {
    if (pro == DG_PRO_PLAIN && epi == DG_EPI_STORE) return launch_rc_m<T, DG_PRO_PLAIN, DG_EPI_STORE>(p, s);
    if (pro == DG_PRO_RMS && epi == DG_EPI_ROPEKV) return launch_rc_m<T, DG_PRO_RMS, DG_EPI_ROPEKV>(p, s);
    if (pro == DG_PRO_RMS && epi == DG_EPI_SWIGLU) return launch_rc_m<T, DG_PRO_RMS, DG_EPI_SWIGLU>(p, s);
    if (pro == DG_PRO_RMS && epi == DG_EPI_ARGMAX) return launch_rc_m<T, DG_PRO_RMS, DG_EPI_ARGMAX>(p, s);
    return set_error(WGB_ERR_INVALID_ARGUMENT, "ref_chain_gemv: prologue %d with epilogue %d", pro, epi);
}

template <typename T> void rc_set_attrs_t() {
#define WGB_RC_ATTR(PRO, EPI)                 \
    rc_set_attr<T, 1, PRO, EPI>();            \
    rc_set_attr<T, 2, PRO, EPI>();            \
    rc_set_attr<T, 4, PRO, EPI>();
    WGB_RC_ATTR(DG_PRO_PLAIN, DG_EPI_STORE)
    WGB_RC_ATTR(DG_PRO_RMS, DG_EPI_ROPEKV)
    WGB_RC_ATTR(DG_PRO_RMS, DG_EPI_SWIGLU)
    WGB_RC_ATTR(DG_PRO_RMS, DG_EPI_ARGMAX)
#undef WGB_RC_ATTR
}

// ---- decode attention --------------------------------------------------------
constexpr int kRaCluster = 8;   // CTAs per (sequence, head)
constexpr int kRaThreads = 128;

template <typename T, int DH> struct RaGeom {
    static constexpr int V = 16 / sizeof(T);
    static constexpr int COLS = DH / kRaCluster;  // output columns per CTA
    static constexpr int VPR = DH / V;            // 16-byte vectors per K row
};

// scores / probabilities [maxlen rounded up to 4] f32, the V column slice
// [maxlen][dh / 8]
__host__ __device__ inline int ra_scores_len(int maxlen) { return (maxlen + 3) & ~3; }
size_t ra_smem_bytes(size_t es, int dh, int maxlen) {
    return (size_t)ra_scores_len(maxlen) * 4 + (size_t)maxlen * (dh / kRaCluster) * es;
}

template <typename T, int DH>
__global__ void __launch_bounds__(kRaThreads) ref_attn_decode_kernel(const T *__restrict__ q, const T *kcache,
                                                                     const T *vcache, size_t seq_stride,
                                                                     const int64_t *lens, T *__restrict__ out, int nh,
                                                                     int nkvh, int maxlen, float scale) {
    using G = RaGeom<T, DH>;
    constexpr int V = G::V, COLS = G::COLS, VPR = G::VPR;
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ float s_red[kRaThreads / 32];
    __shared__ float s_sum;
    cg::cluster_group cluster = cg::this_cluster();
    const int r = (int)cluster.block_rank();
    const int b = blockIdx.y / nh, h = blockIdx.y % nh;
    const int kvh = h / (nh / nkvh);
    const int tid = threadIdx.x;
    float *sc = reinterpret_cast<float *>(smem);                       // [maxlen]
    T *vs = reinterpret_cast<T *>(sc + ra_scores_len(maxlen));         // [maxlen][COLS]

    pdl_trigger();
    // the lengths were set by an earlier step; the cached rows other than
    // the newest were written by earlier steps too, so they are requested
    // before the wait for the previous kernel (which writes q and the newest
    // K/V row)
    long Ll = lens[b] + 1;
    if (Ll > maxlen) Ll = maxlen;
    if (Ll < 1) Ll = 1;
    const int L = (int)Ll, newest = L - 1;
    const size_t rstride = (size_t)nkvh * DH;  // elements between cached positions
    const T *kb = kcache + (size_t)b * seq_stride + (size_t)kvh * DH;
    const T *vb = vcache + (size_t)b * seq_stride + (size_t)kvh * DH + r * COLS;
    // this CTA's V columns, all positions, into shared memory (needed last)
    for (int i = tid; i < L * (COLS / V); i += kRaThreads) {
        const int j = i / (COLS / V), c = i - j * (COLS / V);
        if (j != newest) __pipeline_memcpy_async(vs + (size_t)j * COLS + c * V, vb + (size_t)j * rstride + c * V, 16);
    }
    // scores (self_attention_cpu.cpp:37-45): scale * (sequential dot over d);
    // this CTA's keys are [j0, j1), one key per thread per pass, two passes
    // interleaved, the first pass's key rows loaded before the wait. Every
    // score goes to every CTA of the cluster, which then runs the softmax
    // itself (the same operations in the same order, so the same bits in
    // every CTA): one cluster barrier and no copy of the probabilities.
    float *scr[kRaCluster];
#pragma unroll
    for (int c = 0; c < kRaCluster; c++) scr[c] = cluster.map_shared_rank(sc, c);
    const int per = (L + kRaCluster - 1) / kRaCluster;
    const int j0 = r * per, j1 = min(L, j0 + per);
    uint4 ka[VPR], kbv[VPR];
    auto load_rows = [&](int ja, int jb, bool early) {
#pragma unroll
        for (int u = 0; u < VPR; u++) {
            if (ja < j1 && (ja != newest) == early) ka[u] = *reinterpret_cast<const uint4 *>(kb + (size_t)ja * rstride + u * V);
            if (jb < j1 && (jb != newest) == early) kbv[u] = *reinterpret_cast<const uint4 *>(kb + (size_t)jb * rstride + u * V);
        }
    };
#pragma unroll
    for (int u = 0; u < VPR; u++) ka[u] = kbv[u] = make_uint4(0u, 0u, 0u, 0u);
    load_rows(j0 + tid, j0 + tid + kRaThreads, true);
    pdl_wait();
    for (int i = tid; i < COLS / V; i += kRaThreads)
        if (newest < L) __pipeline_memcpy_async(vs + (size_t)newest * COLS + i * V, vb + (size_t)newest * rstride + i * V, 16);
    __pipeline_commit();
    const uint4 *qrow = reinterpret_cast<const uint4 *>(q + ((size_t)b * nh + h) * DH);
    for (int ja = j0 + tid; ja < j1; ja += 2 * kRaThreads) {
        const int jb = ja + kRaThreads;
        const bool hb = jb < j1;
        if (ja == j0 + tid) {
            load_rows(ja, jb, false);  // the newest row, if it is one of these
        } else {
#pragma unroll
            for (int u = 0; u < VPR; u++) {
                ka[u] = *reinterpret_cast<const uint4 *>(kb + (size_t)ja * rstride + u * V);
                kbv[u] = hb ? *reinterpret_cast<const uint4 *>(kb + (size_t)jb * rstride + u * V)
                            : make_uint4(0u, 0u, 0u, 0u);
            }
        }
        uint4 qv[VPR];
#pragma unroll
        for (int u = 0; u < VPR; u++) qv[u] = qrow[u];
        float aa = 0.f, ab = 0.f;
#pragma unroll
        for (int u = 0; u < VPR; u++) {
            chain_vec<T>(aa, qv[u], ka[u]);
            chain_vec<T>(ab, qv[u], kbv[u]);
        }
        const float sa = __fmul_rn(scale, aa), sb = __fmul_rn(scale, ab);
#pragma unroll
        for (int c = 0; c < kRaCluster; c++) {
            scr[c][ja] = sa;
            if (hb) scr[c][jb] = sb;
        }
    }
    cluster.sync();  // every score is in every CTA; no CTA reads another's shared memory after this

    {
        // softmax (self_attention_cpu.cpp:63-77): max, exp(s - max), a
        // sequential sum over every key, then one division per key
        float mx = -FLT_MAX;
        for (int j = tid; j < L; j += kRaThreads) mx = fmaxf(mx, sc[j]);
        mx = warp_max(mx);
        if ((tid & 31) == 0) s_red[tid >> 5] = mx;
        __syncthreads();
        mx = s_red[0];
        for (int i = 1; i < kRaThreads / 32; i++) mx = fmaxf(mx, s_red[i]);
        for (int j = tid; j < L; j += kRaThreads) sc[j] = expf_glibc(__fsub_rn(sc[j], mx));
        __syncthreads();
        if (tid == 0) {
            float sum = 0.f;
            int j = 0;
            for (; j + 32 <= L; j += 32) {  // 32 operands loaded, then 32 chain steps
                float4 e4[8];
#pragma unroll
                for (int q = 0; q < 8; q++) e4[q] = *reinterpret_cast<const float4 *>(sc + j + 4 * q);
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    sum = __fadd_rn(sum, e4[q].x);
                    sum = __fadd_rn(sum, e4[q].y);
                    sum = __fadd_rn(sum, e4[q].z);
                    sum = __fadd_rn(sum, e4[q].w);
                }
            }
            for (; j < L; j++) sum = __fadd_rn(sum, sc[j]);
            s_sum = sum;
        }
        __syncthreads();
        const float sum = s_sum;
        for (int j = tid; j < L; j += kRaThreads) sc[j] = __fdiv_rn(sc[j], sum);
    }
    __pipeline_wait_prior(0);
    __syncthreads();
    // output (self_attention_cpu.cpp:81-89): per column a sequential sum over
    // keys of round(p * v)
    if (tid < COLS) {
        float acc = 0.f;
        int j = 0;
        const uint32_t sc_s = smem_u32(sc);
        for (; j + 16 <= L; j += 16) {  // 16 keys' operands loaded, then 16 chain steps
            float4 p4[4];
            float vv[16];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint4 w = lds128(sc_s + (uint32_t)((j + 4 * q) * 4));
                p4[q] = make_float4(__uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z),
                                    __uint_as_float(w.w));
            }
#pragma unroll
            for (int u = 0; u < 16; u++) vv[u] = Elem<T>::load(vs[(size_t)(j + u) * COLS + tid]);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                acc = __fadd_rn(acc, __fmul_rn(p4[q].x, vv[4 * q + 0]));
                acc = __fadd_rn(acc, __fmul_rn(p4[q].y, vv[4 * q + 1]));
                acc = __fadd_rn(acc, __fmul_rn(p4[q].z, vv[4 * q + 2]));
                acc = __fadd_rn(acc, __fmul_rn(p4[q].w, vv[4 * q + 3]));
            }
        }
        for (; j < L; j++) acc = __fadd_rn(acc, __fmul_rn(sc[j], Elem<T>::load(vs[(size_t)j * COLS + tid])));
        stf(out, ((size_t)b * nh + h) * DH + r * COLS + tid, acc);
    }
}

template <typename T, int DH> void ra_set_attr() {
    if (cudaFuncSetAttribute(ref_attn_decode_kernel<T, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemLimit) != cudaSuccess)
        cudaGetLastError();
}

template <typename T, int DH>
int launch_ra(T *out, const T *q, const T *kc, const T *vc, size_t seq_stride, const int64_t *lens, int B, int nh,
              int nkvh, int maxlen, float scale, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kRaCluster, (unsigned)(B * nh), 1);
    cfg.blockDim = dim3(kRaThreads, 1, 1);
    cfg.dynamicSmemBytes = ra_smem_bytes(sizeof(T), DH, maxlen);
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kRaCluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    const cudaError_t e =
        cudaLaunchKernelEx(&cfg, ref_attn_decode_kernel<T, DH>, q, kc, vc, seq_stride, lens, out, nh, nkvh, maxlen, scale);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "self_attention(reference decode): %s", cudaGetErrorString(e));
    return check_launch("self_attention(reference decode)");
}

}  // namespace

bool ref_chain_ok(wginferDataType_t dtype, const DecodeGemvParams &p) {
    if (dtype != WGINFER_DTYPE_BF16 && dtype != WGINFER_DTYPE_F16 && dtype != WGINFER_DTYPE_F32) return false;
    const size_t es = dtype == WGINFER_DTYPE_F32 ? 4 : 2;
    if (p.M0 < 1 || p.M0 > kRefChainMaxM || p.N < 1 || p.K < 1) return false;
    if ((p.K * es) % 16 != 0 || !aligned16(p.w) || !aligned16(p.x) || (p.norm_w && !aligned16(p.norm_w)))
        return false;
    const int mt = p.M0 <= 1 ? 1 : p.M0 <= 2 ? 2 : 4;
    return rc_smem_bytes(1, 4, 1, mt, p.K, es) <= kSmemLimit;  // at least a 4-stage ring
}

int ref_chain_gemv(wginferDataType_t dtype, const DecodeGemvParams &p, int pro, int epi, cudaStream_t s) {
    WGB_REQUIRE(ref_chain_ok(dtype, p), WGB_ERR_INVALID_ARGUMENT, "ref_chain_gemv: unsupported shape or alignment");
    switch (dtype) {
    case WGINFER_DTYPE_BF16: return launch_rc_t<__nv_bfloat16>(p, pro, epi, s);
    case WGINFER_DTYPE_F16: return launch_rc_t<__half>(p, pro, epi, s);
    default: return launch_rc_t<float>(p, pro, epi, s);
    }
}

bool ref_attn_decode_ok(wginferDataType_t dtype, int nh, int nkvh, int dh, int maxlen, const void *kcache,
                        const void *vcache, size_t seq_stride) {
    if (dtype != WGINFER_DTYPE_BF16 && dtype != WGINFER_DTYPE_F16 && dtype != WGINFER_DTYPE_F32) return false;
    const size_t es = dtype == WGINFER_DTYPE_F32 ? 4 : 2;
    if ((dh != 128 && dh != 64) || nkvh < 1 || nh % nkvh) return false;
    if (((size_t)(dh / kRaCluster) * es) % 16 != 0) return false;  // whole 16-byte pieces per V row slice
    if (!aligned16(kcache) || !aligned16(vcache) || (seq_stride * es) % 16 != 0 || ((size_t)nkvh * dh * es) % 16 != 0)
        return false;
    return maxlen >= 1 && ra_smem_bytes(es, dh, maxlen) <= kSmemLimit;
}

int ref_attn_decode(wginferDataType_t dtype, void *out, const void *q, const void *kcache, const void *vcache,
                    size_t seq_stride, const int64_t *lens, int B, int nh, int nkvh, int dh, int maxlen, float scale,
                    cudaStream_t s) {
    WGB_REQUIRE(ref_attn_decode_ok(dtype, nh, nkvh, dh, maxlen, kcache, vcache, seq_stride), WGB_ERR_INVALID_ARGUMENT,
                "ref_attn_decode: unsupported shape or alignment");
    WGB_REQUIRE(B >= 1 && (long)B * nh < 65536, WGB_ERR_INVALID_ARGUMENT, "ref_attn_decode: batch %d", B);
#define WGB_RA(TT)                                                                                                   \
    return dh == 128 ? launch_ra<TT, 128>((TT *)out, (const TT *)q, (const TT *)kcache, (const TT *)vcache,          \
                                          seq_stride, lens, B, nh, nkvh, maxlen, scale, s)                           \
                     : launch_ra<TT, 64>((TT *)out, (const TT *)q, (const TT *)kcache, (const TT *)vcache, seq_stride, \
                                         lens, B, nh, nkvh, maxlen, scale, s)
    switch (dtype) {
    case WGINFER_DTYPE_BF16: WGB_RA(__nv_bfloat16);
    case WGINFER_DTYPE_F16: WGB_RA(__half);
    default: WGB_RA(float);
    }
#undef WGB_RA
}

void ref_decode_prepare() {
    static thread_local unsigned long long done_mask = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || ((done_mask >> dev) & 1ull)) return;
    rc_set_attrs_t<__nv_bfloat16>();
    rc_set_attrs_t<__half>();
    rc_set_attrs_t<float>();
    ra_set_attr<__nv_bfloat16, 128>();
    ra_set_attr<__nv_bfloat16, 64>();
    ra_set_attr<__half, 128>();
    ra_set_attr<__half, 64>();
    ra_set_attr<float, 128>();
    ra_set_attr<float, 64>();
    done_mask |= 1ull << dev;
}

}  // namespace wgb
