// Fused decode GEMV for the Qwen2 caller (FAST numerics, bf16/f16/f32).
//
// One weight-streaming kernel per projection, with the neighbouring
// elementwise work folded in so that it costs no extra launch and no extra
// HBM round trip:
//   prologue  RMS   - the input row is rms-normalised inside every CTA (the
//                     row is 3 KB and sits in L2): xn = round(x * w * s),
//                     exactly what a separate rms_norm would write;
//   epilogue  STORE - round(acc + bias), optionally + residual (the skip
//                     connection: round(r + round(acc)), model.cpp:436-463);
//             SWIGLU- the two rows of a warp are gate row j and up row j:
//                     act[j] = round(u * g / (1 + exp(-g))) of the rounded
//                     projections (swiglu_cpu.cpp:11);
//             ROPEKV- the two rows of a warp are rotation partners (j, j+dh/2)
//                     of one q or k head: the rounded pair is rotated with
//                     the host-built cos/sin table and written to q_rope or
//                     straight into the K cache; v rows go to the V cache.
//             ARGMAX- the lm_head of a decode step: logits stored as with
//                     STORE, and each row's greedy token found on the way:
//                     a CTA folds its outputs' (value, first index) keys
//                     (argmax_key.cuh) in shared memory, merges them with one
//                     global atomic per input row, and the CTA that finishes
//                     last writes the tokens and advances the sequence
//                     lengths (model.cpp:398-407), so no argmax launch and
//                     no second pass over the 151936 logits follow.
// Each warp owns two weight rows at a time (chosen by the epilogue's row map)
// and a 1/KS slice of K; lanes stream 16-byte weight vectors with an L2
// evict-first policy, several vectors in flight per lane. The grid is
// persistent (every CTA resident at once) so the prologue runs once per CTA, and each CTA
// prefetches its next block of rows into L2 while it works on the current one.
//
// Launch: programmatic dependent launch. A CTA first prefetches its weight
// rows into L2 (cp.async.bulk.prefetch), which does not depend on the
// previous kernel, then waits for the previous kernel's results
// (griddepcontrol.wait); it allows the next kernel to launch at once
// (griddepcontrol.launch_dependents), so launches and weight fetches overlap
// the previous kernel's tail.
#include <cuda_pipeline.h>

#include <atomic>

#include "argmax_key.cuh"
#include "common.cuh"
#include "decode_common.cuh"
#include "kernels.h"

namespace wgb {
namespace {

constexpr int kRows = 2;       // weight rows per warp
constexpr int kMaxMT = 8;      // input rows per launch
constexpr int kVPL = 6;        // 16-byte vectors in flight per row per lane
constexpr int kCtasPerSM = 4;  // persistent grid: at most 32 resident warps per SM

enum Pro { PRO_PLAIN = DG_PRO_PLAIN, PRO_RMS = DG_PRO_RMS };

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename T, int MT, int KS, int PRO, int EPI>
__global__ void __launch_bounds__(256, (MT <= 2 ? 3 : 2)) decode_gemv_kernel(DecodeGemvParams p) {
    constexpr int V = Vec16<T>::N;
    constexpr int GROUPS = 8 / KS;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *xs = reinterpret_cast<T *>(smem_raw);  // [MT][K] normalised input (PRO_RMS)
    T *nws = xs + (size_t)MT * p.K;           // [K] norm weight (PRO_RMS)
    __shared__ float red[8][kRows][MT];
    __shared__ float s_scale[MT];
    __shared__ float s_part[8][MT];
    __shared__ float s_epi[8][MT][4];  // first block: bias (b0, b1) and residual (q0, q1) per warp and row
    __shared__ unsigned long long s_key[MT];  // ARGMAX: this CTA's best key per input row
    if (EPI == EPI_ARGMAX && threadIdx.x < MT) s_key[threadIdx.x] = 0ull;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = warp / KS, ks = warp % KS;
    const int K = p.K, M = p.M;
    const int nblocks = (p.groups + GROUPS - 1) / GROUPS;

    auto prefetch_block = [&](int blk) {
        const int g = blk * GROUPS + rg;
        if (blk < nblocks && g < p.groups && ks == 0 && lane == 0) {
            int r0, r1;
            row_map<EPI>(p, g, r0, r1);
            prefetch_l2(reinterpret_cast<const T *>(p.w) + (size_t)r0 * K, (uint32_t)(K * sizeof(T)));
            if (r1 < p.N) prefetch_l2(reinterpret_cast<const T *>(p.w) + (size_t)r1 * K, (uint32_t)(K * sizeof(T)));
        }
    };
    const uint64_t pol = evict_first_policy();
    const int nvec = K / V;
    const int per = (nvec + KS - 1) / KS;
    const int v0 = ks * per, v1 = min(v0 + per, nvec);

    // The first block's first chunk of weights is requested before waiting
    // for the previous kernel: weights do not depend on it, so their HBM
    // round trip overlaps that kernel's tail. Later blocks were prefetched
    // into L2 one block ahead.
    Vec16<T> wa[kVPL], wb[kVPL];
    int blk = blockIdx.x;
    bool have = false;  // wa/wb hold the first chunk of block blk
    auto load_chunk = [&](int b, int c0) {
        const int g = b * GROUPS + rg;
        if (g >= p.groups) return;
        int r0, r1;
        row_map<EPI>(p, g, r0, r1);
        const T *w0 = reinterpret_cast<const T *>(p.w) + (size_t)r0 * K;
        const T *w1 = reinterpret_cast<const T *>(p.w) + (size_t)(r1 < p.N ? r1 : r0) * K;
#pragma unroll
        for (int u = 0; u < kVPL; u++) {
            const int vi = c0 + lane + 32 * u;
            if (vi < v1) {
                wa[u].u = ld_stream_v4(w0 + (size_t)vi * V, pol);
                wb[u].u = ld_stream_v4(w1 + (size_t)vi * V, pol);
            }
        }
    };
    if (blk < nblocks) {
        load_chunk(blk, v0);
        have = true;
    }
    prefetch_block(blk + gridDim.x);
    if (threadIdx.x == 0) {  // the next kernels' weights stream into L2 behind this one
        l2_prefetch_share(p.pf_ptr[0], p.pf_bytes[0], blockIdx.x, gridDim.x);
        l2_prefetch_share(p.pf_ptr[1], p.pf_bytes[1], blockIdx.x, gridDim.x);
    }
    // RoPE epilogue: the positions (set at the start of the step) and the
    // host-built cos/sin table do not depend on the previous kernel; the
    // epilogue lanes of the first block fetch their entries now.
    // The bias of the first block's rows is fetched now too (parked in shared
    // memory, not held in registers across the main loop), and the RMS
    // prologue's norm weight is copied into shared memory (cp.async).
    const int g_first = (int)blockIdx.x * GROUPS + rg;
    int r0_first = 0, r1_first = 0;
    if (g_first < p.groups) row_map<EPI>(p, g_first, r0_first, r1_first);
    const bool epi_lane = ks == 0 && lane < M && lane < MT && g_first < p.groups;
    int64_t pos_pre = 0;
    float2 cs_pre = make_float2(0.f, 0.f);
    float b0_pre = 0.f, b1_pre = 0.f;
    if (epi_lane) {
        if (p.bias) {
            b0_pre = ldf(reinterpret_cast<const T *>(p.bias), r0_first);
            if (r1_first < p.N) b1_pre = ldf(reinterpret_cast<const T *>(p.bias), r1_first);
        }
        if (EPI == EPI_ROPEKV) {
            pos_pre = p.pos[lane];
            const int half = p.dh >> 1;
            if (g_first < (p.nh + p.nkvh) * half && pos_pre >= 0 && pos_pre < p.maxseq)
                cs_pre = p.table[(size_t)pos_pre * half + (g_first % half)];
        }
    }
    if (PRO == PRO_RMS) {
        for (int vi = threadIdx.x; vi < nvec; vi += 256)
            __pipeline_memcpy_async(nws + (size_t)vi * V, reinterpret_cast<const T *>(p.norm_w) + (size_t)vi * V, 16);
        __pipeline_commit();
    }
    pdl_trigger();
    if (epi_lane && p.bias) {
        s_epi[warp][lane][0] = b0_pre;
        s_epi[warp][lane][1] = b1_pre;
    }
    pdl_wait();
    // the residual of the first block's outputs (written by earlier kernels)
    if (EPI == EPI_STORE && p.res && epi_lane) {
        const T *res = reinterpret_cast<const T *>(p.res);
        s_epi[warp][lane][2] = ldf(res, (size_t)lane * p.ldo + r0_first);
        if (r1_first < p.N) s_epi[warp][lane][3] = ldf(res, (size_t)lane * p.ldo + r1_first);
    }
    const T *x = reinterpret_cast<const T *>(p.x);
    if (PRO == PRO_RMS) {
        // every (persistent) CTA normalises the few input rows once: one
        // round trip of 16-byte loads (x rows and the norm weight together),
        // raw rows parked in shared memory, a block reduction, then the
        // scaling pass over shared memory
        float ss[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) ss[m] = 0.f;
        for (int vi = threadIdx.x; vi < nvec; vi += 256) {
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if (m < M) {
                    Vec16<T> xv;
                    xv.u = *reinterpret_cast<const uint4 *>(x + (size_t)m * K + (size_t)vi * V);
                    *reinterpret_cast<uint4 *>(xs + (size_t)m * K + (size_t)vi * V) = xv.u;
#pragma unroll
                    for (int e = 0; e < V; e++) {
                        const float f = Elem<T>::load(xv.e[e]);
                        ss[m] = fmaf(f, f, ss[m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) s_part[warp][m] = t;
        }
        __syncthreads();
        if (threadIdx.x < MT) {
            float t = 0.f;
            for (int q = 0; q < 8; q++) t += s_part[q][threadIdx.x];
            const float mean = __fdiv_rn(t, (float)K);
            s_scale[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        }
        __pipeline_wait_prior(0);  // this thread's norm-weight copies have landed
        __syncthreads();
        for (int vi = threadIdx.x; vi < nvec; vi += 256) {
            Vec16<T> wv;
            wv.u = *reinterpret_cast<const uint4 *>(nws + (size_t)vi * V);
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if (m < M) {
                    Vec16<T> xv;
                    uint4 *q = reinterpret_cast<uint4 *>(xs + (size_t)m * K + (size_t)vi * V);
                    xv.u = *q;
                    const float sc = s_scale[m];
#pragma unroll
                    for (int e = 0; e < V; e++)
                        xv.e[e] = Elem<T>::store(
                            __fmul_rn(__fmul_rn(Elem<T>::load(xv.e[e]), Elem<T>::load(wv.e[e])), sc));
                    *q = xv.u;
                }
            }
        }
        __syncthreads();
        x = xs;
    }
    for (; blk < nblocks; blk += gridDim.x) {
        if (blk != (int)blockIdx.x) prefetch_block(blk + gridDim.x);
        const int g = blk * GROUPS + rg;
        const bool gok = g < p.groups;
        int r0 = 0, r1 = 0;
        if (gok) row_map<EPI>(p, g, r0, r1);
        const bool r1ok = gok && r1 < p.N;

        float acc[kRows][MT];
#pragma unroll
        for (int r = 0; r < kRows; r++)
#pragma unroll
            for (int m = 0; m < MT; m++) acc[r][m] = 0.f;
        if (gok) {
            // all of a lane's vectors for both rows are requested before any
            // is used: up to kVPL per row in one round trip
            for (int c0 = v0; c0 < v1; c0 += 32 * kVPL) {
                if (!have) load_chunk(blk, c0);
                have = false;
#pragma unroll
                for (int u = 0; u < kVPL; u++) {
                    const int vi = c0 + lane + 32 * u;
                    if (vi < v1) {
#pragma unroll
                        for (int m = 0; m < MT; m++) {
                            if (m < M) {
                                Vec16<T> xv;
                                xv.u = *reinterpret_cast<const uint4 *>(x + (size_t)m * K + (size_t)vi * V);
#pragma unroll
                                for (int e = 0; e < V; e++) {
                                    const float xf = Elem<T>::load(xv.e[e]);
                                    acc[0][m] = fmaf(xf, Elem<T>::load(wa[u].e[e]), acc[0][m]);
                                    acc[1][m] = fmaf(xf, Elem<T>::load(wb[u].e[e]), acc[1][m]);
                                }
                            }
                        }
                    }
                }
            }
        }
        // the next block's first chunk is requested now (an L2 hit: it was
        // prefetched a block ago), so its round trip overlaps this block's
        // reduction and epilogue
        have = false;
        if (blk + (int)gridDim.x < nblocks) {
            load_chunk(blk + gridDim.x, v0);
            have = true;
        }
#pragma unroll
        for (int r = 0; r < kRows; r++)
#pragma unroll
            for (int m = 0; m < MT; m++) acc[r][m] = warp_sum(acc[r][m]);
        if (KS > 1) {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < kRows; r++)
#pragma unroll
                    for (int m = 0; m < MT; m++) red[warp][r][m] = acc[r][m];
            }
            __syncthreads();
        }
        if (gok && ks == 0 && lane < MT && lane < M) {
            const int m = lane;
            float s0 = 0.f, s1 = 0.f;
            if (KS > 1) {
                for (int q = 0; q < KS; q++) {
                    s0 += red[warp + q][0][m];
                    s1 += red[warp + q][1][m];
                }
            } else {
#pragma unroll
                for (int mm = 0; mm < MT; mm++)
                    if (mm == m) {
                        s0 = acc[0][mm];
                        s1 = acc[1][mm];
                    }
            }
            if (EPI == EPI_ARGMAX) {
                T *out = reinterpret_cast<T *>(p.out);
                stf(out, (size_t)m * p.ldo + r0, s0);
                unsigned long long k = key_or_zero(Elem<T>::load(Elem<T>::store(s0)), (uint32_t)r0);
                if (r1ok) {
                    stf(out, (size_t)m * p.ldo + r1, s1);
                    const unsigned long long k1 = key_or_zero(Elem<T>::load(Elem<T>::store(s1)), (uint32_t)r1);
                    k = k1 > k ? k1 : k;
                }
                if (k) atomicMax(&s_key[m], k);
            } else if (blk == (int)blockIdx.x) {
                EpiPre pre;
                if (p.bias) {
                    pre.b0 = s_epi[warp][m][0];
                    pre.b1 = s_epi[warp][m][1];
                }
                if (EPI == EPI_STORE && p.res) {
                    pre.q0 = s_epi[warp][m][2];
                    pre.q1 = r1ok ? s_epi[warp][m][3] : 0.f;
                }
                pre.pos = pos_pre;
                pre.cs = cs_pre;
                epilogue_pre<T, EPI>(p, g, r0, r1, r1ok, m, s0, s1, pre);
            } else
                epilogue<T, EPI>(p, g, r0, r1, r1ok, m, s0, s1);
        }
        if (KS > 1) __syncthreads();  // red[] is rewritten by the next block
    }
    if (EPI == EPI_ARGMAX) {
        __syncthreads();
        if (threadIdx.x < M && s_key[threadIdx.x]) {
            atomicMax(&p.amax_keys[threadIdx.x], s_key[threadIdx.x]);
            __threadfence();
        }
        __syncthreads();
        // the CTA that finishes last turns the keys into tokens
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned done = atomicAdd(p.amax_count, 1u);
            if (done == gridDim.x - 1) {
                __threadfence();
                for (int m = 0; m < M; m++) {
                    const unsigned long long key = atomicExch(&p.amax_keys[m], 0ull);
                    const T *row0 = reinterpret_cast<const T *>(p.out) + (size_t)m * p.ldo;
                    T x0;
                    if constexpr (sizeof(T) == 4) {
                        x0 = __ldcg(reinterpret_cast<const float *>(row0));
                    } else {
                        const unsigned short u = __ldcg(reinterpret_cast<const unsigned short *>(row0));
                        memcpy(&x0, &u, 2);
                    }
                    p.tokens[m] = key_index(key, Elem<T>::load(x0));
                    if (p.lens && p.lens[m] < p.maxlen) p.lens[m] += 1;
                }
                atomicExch(p.amax_count, 0u);
            }
        }
    }
}

// Resident CTAs of 256 threads per SM for one kernel variant with `smem`
// dynamic shared memory, cached per device and variant (the answer depends
// only on the kernel's resources); at least 1.
template <typename T, int MT, int KS, int PRO, int EPI>
int resident_ctas(size_t smem) {
    static std::atomic<unsigned long long> cache[64];  // [device] -> (smem + 1) << 8 | ctas
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long key = (unsigned long long)(smem + 1) << 8;
    if (dev >= 0 && dev < 64) {
        const unsigned long long c = cache[dev].load(std::memory_order_relaxed);
        if ((c & ~0xFFull) == key) return (int)(c & 0xFF);
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_gemv_kernel<T, MT, KS, PRO, EPI>, 256, smem) !=
            cudaSuccess ||
        n < 1) {
        cudaGetLastError();
        n = 1;
    }
    n = n > kCtasPerSM ? kCtasPerSM : n;
    if (dev >= 0 && dev < 64) cache[dev].store(key | (unsigned long long)n, std::memory_order_relaxed);
    return n;
}

template <typename T, int MT, int KS, int PRO, int EPI>
int launch_one(const DecodeGemvParams &p, cudaStream_t s) {
    constexpr int GROUPS = 8 / KS;
    const int nblocks = (p.groups + GROUPS - 1) / GROUPS;
    const size_t smem = PRO == PRO_RMS ? (size_t)(MT + 1) * p.K * sizeof(T) : 0;
    // persistent: as many CTAs as can be resident at once (registers decide:
    // 72-116 per thread give 2-3 CTAs of 256 threads per SM), each looping
    // over weight-row blocks, so no CTA waits for another to retire
    const int cap = sm_count() * resident_ctas<T, MT, KS, PRO, EPI>(smem);
    const int blocks = nblocks < cap ? nblocks : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, decode_gemv_kernel<T, MT, KS, PRO, EPI>, p);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "decode_gemv: %s", cudaGetErrorString(e));
    return WGB_OK;
}

// K split across KS warps: enough that a lane's share of a row fits one
// round trip (<= kVPL vectors), and more while the grid would leave SMs idle.
template <typename T, int MT, int PRO, int EPI>
int launch_ks(const DecodeGemvParams &p, cudaStream_t s) {
    const int nvec = p.K / Vec16<T>::N;
    int ks = 1;
    while (ks < 8 && (nvec + ks - 1) / ks > 32 * kVPL) ks *= 2;
    while (ks < 8 && (p.groups + 8 / ks - 1) / (8 / ks) < 2 * sm_count() && (nvec + 2 * ks - 1) / (2 * ks) >= 32)
        ks *= 2;
    // ... but not past the point where the blocks no longer fit in one wave
    // of resident CTAs when half the split would: a second wave costs a
    // whole extra round trip for most CTAs, more than a second chunk of each
    // lane's slice (down projection at batch 1: K split 4 with two chunks
    // measured 3.6% faster per decode step than split 8 in 1.7 waves)
    const size_t smem = PRO == PRO_RMS ? (size_t)(MT + 1) * p.K * sizeof(T) : 0;
    const int ctas = sm_count() * resident_ctas<T, MT, 8, PRO, EPI>(smem);
    auto blocks = [&](int k) { return (p.groups + 8 / k - 1) / (8 / k); };
    while (ks > 1 && blocks(ks) > ctas && blocks(ks / 2) <= ctas && (nvec + ks / 2 - 1) / (ks / 2) <= 2 * 32 * kVPL)
        ks /= 2;
    switch (ks) {
    case 1: return launch_one<T, MT, 1, PRO, EPI>(p, s);
    case 2: return launch_one<T, MT, 2, PRO, EPI>(p, s);
    case 4: return launch_one<T, MT, 4, PRO, EPI>(p, s);
    default: return launch_one<T, MT, 8, PRO, EPI>(p, s);
    }
}

template <typename T, int PRO, int EPI>
int launch_mt(const DecodeGemvParams &p, cudaStream_t s) {
    if (p.M <= 1) return launch_ks<T, 1, PRO, EPI>(p, s);
    if (p.M <= 2) return launch_ks<T, 2, PRO, EPI>(p, s);
    if (p.M <= 4) return launch_ks<T, 4, PRO, EPI>(p, s);
    return launch_ks<T, 8, PRO, EPI>(p, s);
}

template <typename T>
int dispatch(const DecodeGemvParams &p0, int pro, int epi, cudaStream_t s) {
    WGB_REQUIRE(p0.K > 0 && p0.K % Vec16<T>::N == 0, WGB_ERR_INVALID_ARGUMENT,
                "decode_gemv: K = %d is not a whole number of 16-byte vectors", p0.K);
    // more than 8 rows of bf16: one tensor-core GEMM over all rows (the RMS
    // prologue first materialised into p0.xn)
    if (std::is_same<T, __nv_bfloat16>::value && p0.M0 > kMaxMT && (pro == PRO_PLAIN || p0.xn)) {
        DecodeGemvParams p = p0;
        p.M = p0.M0;
        if (pro == PRO_RMS) p.x = p0.xn;
        if (tc_gemm_ok(p)) {
            if (pro == PRO_RMS) {
                const int rc = wgb_rms_norm(p0.xn, p0.x, p0.norm_w, WGINFER_DTYPE_BF16, p0.M0, p0.K, p0.eps, s);
                if (rc) return rc;
            }
            return tc_gemm(p, epi, s);
        }
    }
    WGB_REQUIRE(epi != EPI_ARGMAX || p0.M0 <= kMaxMT, WGB_ERR_UNSUPPORTED,
                "decode_gemv: argmax epilogue over %d rows needs bf16 and the tensor-core path", p0.M0);
    // chunks of up to 8 input rows; each chunk re-reads the weights
    for (int m0 = 0; m0 < p0.M0; m0 += kMaxMT) {
        DecodeGemvParams p = p0;
        p.M = min(kMaxMT, p0.M0 - m0);
        p.x = reinterpret_cast<const T *>(p0.x) + (size_t)m0 * p0.K;
        if (p.out) p.out = reinterpret_cast<T *>(p0.out) + (size_t)m0 * p0.ldo;
        if (p.res) p.res = reinterpret_cast<const T *>(p0.res) + (size_t)m0 * p0.ldo;
        if (p.q_out) p.q_out = reinterpret_cast<T *>(p0.q_out) + (size_t)m0 * p0.nh * p0.dh;
        if (p.pos) p.pos = p0.pos + m0;
        if (p0.prefill_seq < 0) {  // row m is sequence m: shift the cache base
            if (p.kc) p.kc = reinterpret_cast<T *>(p0.kc) + (size_t)m0 * p0.seq_stride;
            if (p.vc) p.vc = reinterpret_cast<T *>(p0.vc) + (size_t)m0 * p0.seq_stride;
        }
        int rc;
        if (pro == PRO_RMS && epi == EPI_SWIGLU) rc = launch_mt<T, PRO_RMS, EPI_SWIGLU>(p, s);
        else if (pro == PRO_RMS && epi == EPI_ROPEKV) rc = launch_mt<T, PRO_RMS, EPI_ROPEKV>(p, s);
        else if (pro == PRO_RMS && epi == EPI_STORE) rc = launch_mt<T, PRO_RMS, EPI_STORE>(p, s);
        else if (pro == PRO_PLAIN && epi == EPI_STORE) rc = launch_mt<T, PRO_PLAIN, EPI_STORE>(p, s);
        else if (pro == PRO_RMS && epi == EPI_ARGMAX) {
            // one launch covers every row (the keys are per row of this launch);
            // the K split stays 1 (the lm_head has row blocks to fill the GPU)
            WGB_REQUIRE(p0.M0 <= kMaxMT && !p0.bias && p0.amax_keys && p0.amax_count && p0.tokens,
                        WGB_ERR_INVALID_ARGUMENT, "decode_gemv: argmax epilogue needs <= 8 rows, its key buffers, no bias");
            if (p.M <= 1) rc = launch_one<T, 1, 1, PRO_RMS, EPI_ARGMAX>(p, s);
            else if (p.M <= 2) rc = launch_one<T, 2, 1, PRO_RMS, EPI_ARGMAX>(p, s);
            else if (p.M <= 4) rc = launch_one<T, 4, 1, PRO_RMS, EPI_ARGMAX>(p, s);
            else rc = launch_one<T, 8, 1, PRO_RMS, EPI_ARGMAX>(p, s);
        } else return set_error(WGB_ERR_UNSUPPORTED, "decode_gemv: prologue %d with epilogue %d", pro, epi);
        if (rc) return rc;
    }
    return WGB_OK;
}

template <typename T, int MT, int PRO, int EPI> void attrs_ks() {
    const int lim = 200 * 1024;
    cudaFuncSetAttribute(decode_gemv_kernel<T, MT, 1, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(decode_gemv_kernel<T, MT, 2, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(decode_gemv_kernel<T, MT, 4, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(decode_gemv_kernel<T, MT, 8, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
}
template <typename T, int PRO, int EPI> void attrs_mt() {
    attrs_ks<T, 1, PRO, EPI>();
    attrs_ks<T, 2, PRO, EPI>();
    attrs_ks<T, 4, PRO, EPI>();
    attrs_ks<T, 8, PRO, EPI>();
}
template <typename T> void attrs_all() {
    attrs_mt<T, PRO_RMS, EPI_SWIGLU>();
    attrs_mt<T, PRO_RMS, EPI_ROPEKV>();
    attrs_mt<T, PRO_RMS, EPI_STORE>();
    attrs_mt<T, PRO_PLAIN, EPI_STORE>();
    const int lim = 200 * 1024;
    cudaFuncSetAttribute(decode_gemv_kernel<T, 1, 1, PRO_RMS, EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(decode_gemv_kernel<T, 2, 1, PRO_RMS, EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(decode_gemv_kernel<T, 4, 1, PRO_RMS, EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(decode_gemv_kernel<T, 8, 1, PRO_RMS, EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
}

}  // namespace

void decode_gemv_prepare() {
    tc_gemm_prepare();
    attrs_all<float>();
    attrs_all<__nv_bfloat16>();
    attrs_all<__half>();
}

int decode_gemv(wginferDataType_t dtype, const DecodeGemvParams &p, int pro, int epi, cudaStream_t s) {
    // 16-byte vectors throughout: weights, input rows and the norm weight
    WGB_REQUIRE(aligned16(p.w) && aligned16(p.x) && (pro != PRO_RMS || aligned16(p.norm_w)), WGB_ERR_INVALID_ARGUMENT,
                "decode_gemv: operands must be 16-byte aligned");
    WGB_DISPATCH_FLOAT(dtype, T, return dispatch<T>(p, pro, epi, s));
    return WGB_OK;
}

}  // namespace wgb
