// self_attention: causal GQA attention over a KV cache.
//
// FAST (flash-decode, split-K over a thread-block cluster): a cluster of up
// to 8 CTAs owns one query row and a block of HPC heads that share one kv
// head; each CTA takes one slice of the visible keys. K/V tiles of kKT keys
// stream into shared memory with cp.async (double-buffered) and are used once
// for all HPC heads (GQA reuse); scores use an online softmax in f32. The
// slices then meet in distributed shared memory: CTA 0 of the cluster reads
// the others' (max, sum, unnormalised output) and writes the normalised row,
// so there is no workspace and no second launch. The slice count adapts to
// each row's visible length, so a decode graph captured once stays balanced
// as the caches grow. Roofline at decode: HBM,
// (S*nh*d + 2*L*nkvh*d + S*nh*dv) * size bytes.
//
// REFERENCE: one CTA per (query, head) reproduces
// src/ops/self_attention/cpu/self_attention_cpu.cpp:35-89 step for step:
// sequential dot products, -1e9 for masked keys, max, exp, a sequential sum
// over every key, division, and a sequential sum over keys of the rounded
// products p * v. K and V stream through shared memory in chunks so that the
// serial chains read at shared-memory latency.
#include <cooperative_groups.h>
#include <cuda_pipeline.h>
#include <float.h>

#include <type_traits>

#include "common.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace wgb {
namespace {

constexpr int kKT = 64;        // keys per shared-memory tile (FAST)
constexpr int kThreads = 256;
constexpr int kMaxAcc = 8;     // output accumulators per thread (HPC*dv <= 2048)
constexpr int kMaxCluster = 8; // portable cluster size
constexpr int kRefChunk = 128; // keys per shared-memory chunk (REFERENCE)
constexpr int kRefSmemScores = 11000;  // scores kept in shared memory (REFERENCE)

struct AttnShape {
    int S, nh, nkvh, d, dv, L, hpc, nsplit;
    float scale;
};

// Where the keys of query row i live and how many it sees.
//
// KvDense: the op surface. k/v are [L, nkvh, d]; query i sees keys
// j <= i + (L - S). Fully masked rows (L < S) get the reference's uniform
// weights over all L keys.
template <typename T> struct KvDense {
    const T *k, *v;
    __device__ __forceinline__ void row(const AttnShape &sh, int i, const T *&kr, const T *&vr, int &nkeys,
                                        int &nvis, bool &uniform) const {
        kr = k;
        vr = v;
        nkeys = sh.L;
        long last = (long)i + (long)sh.L - (long)sh.S;
        if (last < 0) {
            nvis = sh.L;
            uniform = true;
        } else {
            nvis = (int)(last + 1 < sh.L ? last + 1 : sh.L);
            uniform = false;
        }
    }
};

// KvCache: batched decode. Query row b is the newest token of sequence b,
// whose cache holds lens[b] + 1 positions (its own K/V included); it sees
// all of them.
template <typename T> struct KvCache {
    const T *k, *v;          // cache of sequence 0
    size_t seq_stride;       // elements between consecutive sequences
    const int64_t *lens;     // [B] positions cached before this token
    __device__ __forceinline__ void row(const AttnShape &sh, int b, const T *&kr, const T *&vr, int &nkeys,
                                        int &nvis, bool &uniform) const {
        kr = k + (size_t)b * seq_stride;
        vr = v + (size_t)b * seq_stride;
        long n = lens[b] + 1;
        if (n > sh.L) n = sh.L;  // never beyond the cache capacity
        if (n < 1) n = 1;
        nkeys = (int)n;
        nvis = (int)n;
        uniform = false;
    }
};

// Copies rows [0, nrows) of a [rows][width] tile (row r at src + r * gstride
// elements) into shared memory with row stride sstride elements. kVec: 16-byte
// cp.async chunks (width * size and both strides 16-byte multiples, src
// 16-byte aligned); otherwise element copies.
template <typename T, bool kVec>
__device__ __forceinline__ void load_tile(T *dst, const T *src, int nrows, int width, size_t gstride, int sstride) {
    if (kVec) {
        constexpr int V = 16 / sizeof(T);
        const int cpr = width / V;
        for (int c = threadIdx.x; c < nrows * cpr; c += kThreads) {
            const int r = c / cpr, cc = c - r * cpr;
            __pipeline_memcpy_async(dst + (size_t)r * sstride + cc * V, src + (size_t)r * gstride + cc * V, 16);
        }
    } else {
        for (int c = threadIdx.x; c < nrows * width; c += kThreads) {
            const int r = c / width, cc = c - r * width;
            dst[(size_t)r * sstride + cc] = src[(size_t)r * gstride + cc];
        }
    }
}

struct FastSmem {
    int qs, kt, vt, ps, stat, xml, xo, bytes;  // byte offsets
};

__host__ __device__ inline int pad_row(int width, int es) { return width + 16 / es; }

__host__ __device__ inline FastSmem fast_smem(const AttnShape &sh, int es) {
    FastSmem f;
    int o = 0;
    f.qs = o; o += sh.hpc * sh.d * 4;
    o = (o + 15) & ~15;
    f.kt = o; o += 2 * kKT * pad_row(sh.d, es) * es;
    f.vt = o; o += 2 * kKT * pad_row(sh.dv, es) * es;
    f.ps = o; o += sh.hpc * kKT * 4;
    f.stat = o; o += 3 * 8 * 4;           // m, l, corr for up to 8 heads
    f.xml = o; o += 2 * kMaxCluster * 8 * 4;               // every slice's (m, l) per head, on CTA 0
    f.xo = o; o += sh.nsplit * sh.hpc * sh.dv * 4;         // every slice's partial output, on CTA 0
    f.bytes = o;
    return f;
}

template <typename T, class Src, bool kVec>
__global__ void __launch_bounds__(kThreads) attn_fast_kernel(const T *__restrict__ q, Src src, T *__restrict__ out,
                                                             AttnShape sh) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int es = sizeof(T);
    const FastSmem lay = fast_smem(sh, es);
    float *qs = reinterpret_cast<float *>(smem + lay.qs);
    T *kt = reinterpret_cast<T *>(smem + lay.kt);
    T *vt = reinterpret_cast<T *>(smem + lay.vt);
    float *ps = reinterpret_cast<float *>(smem + lay.ps);
    float *mrow = reinterpret_cast<float *>(smem + lay.stat);
    float *lrow = mrow + 8, *corr = mrow + 16;
    float *xm = reinterpret_cast<float *>(smem + lay.xml);  // [kMaxCluster][8]
    float *xl = xm + kMaxCluster * 8;                        // [kMaxCluster][8]
    float *xo = reinterpret_cast<float *>(smem + lay.xo);    // [nsplit][hpc * dv]
    const int kst = pad_row(sh.d, es), vst = pad_row(sh.dv, es);

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int nsplit = (int)cluster.num_blocks();
    const int hblocks = sh.nh / sh.hpc;
    const int i = blockIdx.y / hblocks;
    const int h0 = (blockIdx.y % hblocks) * sh.hpc;
    const int kvh = h0 * sh.nkvh / sh.nh;
    const int tid = threadIdx.x;
    pdl_trigger();
    pdl_wait();  // q and the cache are written by the previous kernel
    const T *k, *v;
    int nkeys, nvis;
    bool uniform;
    src.row(sh, i, k, v, nkeys, nvis, uniform);
    const int tiles = (nvis + kKT - 1) / kKT;
    const int per = (tiles + nsplit - 1) / nsplit;
    const int j0 = min(rank * per * kKT, nvis), j1 = min((rank + 1) * per * kKT, nvis);
    const size_t kstride = (size_t)sh.nkvh * sh.d, vstride = (size_t)sh.nkvh * sh.dv;
    const T *kb = k + (size_t)kvh * sh.d, *vb = v + (size_t)kvh * sh.dv;

    for (int x = tid; x < sh.hpc * sh.d; x += kThreads) {
        const int hh = x / sh.d, c = x - hh * sh.d;
        qs[x] = ldf(q, ((size_t)i * sh.nh + h0 + hh) * sh.d + c);
    }
    if (tid < sh.hpc) {
        mrow[tid] = -FLT_MAX;
        lrow[tid] = 0.f;
    }
    float acc[kMaxAcc];
#pragma unroll
    for (int a = 0; a < kMaxAcc; a++) acc[a] = 0.f;
    const int nacc = sh.hpc * sh.dv;
    const int kgroups = nacc >= kThreads ? 1 : kThreads / nacc;  // key groups per output column

    auto issue = [&](int t0, int buf) {
        const int nt = min(kKT, j1 - t0);
        load_tile<T, kVec>(kt + (size_t)buf * kKT * kst, kb + (size_t)t0 * kstride, nt, sh.d, kstride, kst);
        load_tile<T, kVec>(vt + (size_t)buf * kKT * vst, vb + (size_t)t0 * vstride, nt, sh.dv, vstride, vst);
        __pipeline_commit();
    };
    if (j0 < j1) issue(j0, 0);
    int buf = 0;
    for (int t0 = j0; t0 < j1; t0 += kKT, buf ^= 1) {
        const int nt = min(kKT, j1 - t0);
        if (t0 + kKT < j1) {
            issue(t0 + kKT, buf ^ 1);
            __pipeline_wait_prior(1);
        } else {
            __pipeline_wait_prior(0);
        }
        __syncthreads();
        const T *K = kt + (size_t)buf * kKT * kst;
        const T *Vt = vt + (size_t)buf * kKT * vst;
        // scores: 4 threads per key, each a quarter of the dot for every head
        {
            const int jj = tid >> 2, qd = tid & 3;
            float part[8];
#pragma unroll
            for (int hh = 0; hh < 8; hh++) part[hh] = 0.f;
            if (jj < nt && !uniform) {
                const int q0 = qd * (sh.d / 4), q1 = (qd == 3) ? sh.d : q0 + sh.d / 4;
                const T *kr = K + (size_t)jj * kst;
                for (int c = q0; c < q1; c++) {
                    const float kv = Elem<T>::load(kr[c]);
#pragma unroll
                    for (int hh = 0; hh < 8; hh++)
                        if (hh < sh.hpc) part[hh] = fmaf(qs[hh * sh.d + c], kv, part[hh]);
                }
            }
#pragma unroll
            for (int hh = 0; hh < 8; hh++) {
                part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], 1);
                part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], 2);
            }
            if (qd == 0 && jj < kKT) {
#pragma unroll
                for (int hh = 0; hh < 8; hh++)
                    if (hh < sh.hpc) ps[hh * kKT + jj] = jj < nt ? (uniform ? 0.f : sh.scale * part[hh]) : -FLT_MAX;
            }
        }
        __syncthreads();
        // online softmax: one warp per head, two keys per lane
        {
            const int warp = tid >> 5, lane = tid & 31;
            for (int hh = warp; hh < sh.hpc; hh += kThreads / 32) {
                const float s0 = ps[hh * kKT + lane], s1 = ps[hh * kKT + lane + 32];
                const float mt = warp_max(fmaxf(s0, s1));
                const float mold = mrow[hh];
                const float mnew = fmaxf(mold, mt);
                const float p0 = lane < nt ? __expf(s0 - mnew) : 0.f;
                const float p1 = lane + 32 < nt ? __expf(s1 - mnew) : 0.f;
                ps[hh * kKT + lane] = p0;
                ps[hh * kKT + lane + 32] = p1;
                const float sp = warp_sum(p0 + p1);
                if (lane == 0) {
                    const float c = __expf(mold - mnew);
                    corr[hh] = c;
                    lrow[hh] = lrow[hh] * c + sp;
                    mrow[hh] = mnew;
                }
            }
        }
        __syncthreads();
        // P.V: when hpc*dv < threads, kgroups threads share a column, each
        // taking every kgroups-th key; their partials meet after the last tile
#pragma unroll
        for (int a = 0; a < kMaxAcc; a++) {
            const int x = tid + a * kThreads;
            if (x < nacc * kgroups) {
                const int col = x % nacc, grp = x / nacc;
                const int hh = col / sh.dv, c = col - hh * sh.dv;
                float sacc = acc[a] * corr[hh];
                const float *pp = ps + hh * kKT;
                const T *vc = Vt + c;
#pragma unroll 4
                for (int jj = grp; jj < nt; jj += kgroups) sacc = fmaf(pp[jj], Elem<T>::load(vc[(size_t)jj * vst]), sacc);
                acc[a] = sacc;
            }
        }
        __syncthreads();
    }
    if (kgroups > 1) {  // fold the key groups: group 0 keeps the column sums
        float *fold = reinterpret_cast<float *>(smem + lay.kt);  // the K tile buffer is free now
#pragma unroll
        for (int a = 0; a < kMaxAcc; a++) {
            const int x = tid + a * kThreads;
            if (x < nacc * kgroups && x >= nacc) fold[x] = acc[a];
        }
        __syncthreads();
#pragma unroll
        for (int a = 0; a < kMaxAcc; a++) {
            const int x = tid + a * kThreads;
            if (x < nacc)
                for (int gidx = 1; gidx < kgroups; gidx++) acc[a] += fold[x + gidx * nacc];
        }
    }
    // publish this slice into CTA 0's shared memory (remote stores do not
    // stall), then CTA 0 folds the slices from its own shared memory
    if (j0 >= j1 && tid < sh.hpc) {
        mrow[tid] = -FLT_MAX;
        lrow[tid] = 0.f;
    }
    __syncthreads();
    {
        float *dxo = cluster.map_shared_rank(xo, 0) + (size_t)rank * nacc;
#pragma unroll
        for (int a = 0; a < kMaxAcc; a++) {
            const int x = tid + a * kThreads;
            if (x < nacc) dxo[x] = acc[a];
        }
        if (tid < sh.hpc) {
            cluster.map_shared_rank(xm, 0)[rank * 8 + tid] = mrow[tid];
            cluster.map_shared_rank(xl, 0)[rank * 8 + tid] = lrow[tid];
        }
    }
    cluster.sync();
    if (rank == 0) {
        for (int x = tid; x < nacc; x += kThreads) {
            const int hh = x / sh.dv, c = x - hh * sh.dv;
            float M = -FLT_MAX;
            for (int r = 0; r < nsplit; r++) M = fmaxf(M, xm[r * 8 + hh]);
            float L = 0.f, O = 0.f;
            for (int r = 0; r < nsplit; r++) {
                const float l = xl[r * 8 + hh];
                if (l > 0.f) {
                    const float w = __expf(xm[r * 8 + hh] - M);
                    L += l * w;
                    O += xo[(size_t)r * nacc + x] * w;
                }
            }
            stf(out, ((size_t)i * sh.nh + h0 + hh) * sh.dv + c, L > 0.f ? O / L : 0.f);
        }
    }
}

// ---- FAST, one head per warp (decode and short query blocks) ---------------
// Lane j of a warp owns key j of a 32-key chunk: its K row (DH elements) is
// loaded into registers and the dot product runs from registers, so the
// score phase has no shared-memory traffic and no block barrier. The same
// lane copies its V row into the warp's shared-memory buffer with cp.async,
// so K and V of a chunk arrive in one round trip. The warp folds the chunk
// into its running (max, sum, output) with shuffles; for P.V each lane owns
// DH/32 output columns and reads the V rows from shared memory. Warps of a
// CTA take interleaved chunks of the CTA's key slice; the NW warps, then the
// cluster's CTAs, are folded in shared memory (pushed into CTA 0).
//
// Over a KV cache (kPre) every row but the newest was written by an earlier
// step, so a warp's first chunk (K into registers, V into shared memory) is
// requested before griddepcontrol.wait; the newest row follows the wait.
constexpr int kWarpKeys = 32;

template <class Src> struct IsKvCache { static constexpr bool value = false; };
template <typename T> struct IsKvCache<KvCache<T>> { static constexpr bool value = true; };

template <typename T, int DH, int NW> constexpr size_t warp_attn_smem() { return (size_t)NW * kWarpKeys * DH * sizeof(T); }

template <typename T, int DH, class Src, int NW>
__global__ void __launch_bounds__(NW * 32) attn_warp_kernel(const T *__restrict__ q, Src src, T *__restrict__ out, AttnShape sh,
                                                             const void *pf_ptr, size_t pf_bytes) {
    constexpr bool kPre = IsKvCache<Src>::value;
    constexpr int V = 16 / sizeof(T);        // elements per 16-byte vector
    constexpr int NV = DH / V;                // vectors per row
    constexpr int CPL = DH / 32;              // output columns per lane
    extern __shared__ __align__(16) unsigned char vsm[];  // [NW warps][32 keys][DH] V rows
    __shared__ __align__(16) float qs[DH];
    __shared__ float wm[NW], wl[NW];
    __shared__ __align__(16) float wo[NW][DH];
    __shared__ float xm[kMaxCluster], xl[kMaxCluster];
    __shared__ __align__(16) float xo[kMaxCluster][DH];

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int nsplit = (int)cluster.num_blocks();
    const int i = blockIdx.y / sh.nh, h = blockIdx.y % sh.nh;
    const int kvh = h * sh.nkvh / sh.nh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T *k, *v;
    int nkeys, nvis;
    bool uniform;
    src.row(sh, i, k, v, nkeys, nvis, uniform);  // lengths were set by an earlier step
    const int chunks = (nvis + kWarpKeys - 1) / kWarpKeys;
    const int per = (chunks + nsplit - 1) / nsplit;
    const int c0 = rank * per, c1 = min(c0 + per, chunks);
    const size_t kst = (size_t)sh.nkvh * DH;
    const T *kb = k + (size_t)kvh * DH, *vb = v + (size_t)kvh * DH;
    T *vs = reinterpret_cast<T *>(vsm) + (size_t)warp * kWarpKeys * DH;  // this warp's V rows
    const int newest = kPre ? nvis - 1 : -1;  // written by the previous kernel

    Vec16<T> kv[NV];
    // lane's key j of chunk ch: K row into registers, V row into shared memory
    auto fetch = [&](int ch) {
        const int j = ch * kWarpKeys + lane;
        if (j < nvis) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(kb + (size_t)j * kst);
#pragma unroll
            for (int u = 0; u < NV; u++) kv[u].u = kr[u];
#pragma unroll
            for (int u = 0; u < NV; u++)
                __pipeline_memcpy_async(vs + (size_t)lane * DH + u * V, vb + (size_t)j * kst + u * V, 16);
        }
        __pipeline_commit();
    };
    const int first = c0 + warp;
    if (kPre && first < c1 && first * kWarpKeys + lane != newest) fetch(first);
    if (threadIdx.x == 32)  // the next kernel's weights stream into L2 meanwhile
        l2_prefetch_share(pf_ptr, pf_bytes, blockIdx.x + gridDim.x * blockIdx.y, gridDim.x * gridDim.y);
    pdl_trigger();
    pdl_wait();  // q and the newest cache row are written by the previous kernel
    if (first < c1 && (!kPre || first * kWarpKeys + lane == newest)) fetch(first);
    for (int c = threadIdx.x; c < DH; c += NW * 32) qs[c] = ldf(q, ((size_t)i * sh.nh + h) * DH + c);
    __syncthreads();

    float m = -FLT_MAX, l = 0.f;
    float o[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) o[c] = 0.f;

    for (int ch = first; ch < c1; ch += NW) {
        if (ch != first) fetch(ch);
        const int j = ch * kWarpKeys + lane;
        const bool ok = j < nvis;
        float sc = -FLT_MAX;
        if (ok) {
            // four independent chains: the dot is latency-bound, not FMA-bound
            float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int u = 0; u < NV; u++)
#pragma unroll
                for (int e = 0; e < V; e++)
                    d4[(u * V + e) & 3] = fmaf(qs[u * V + e], Elem<T>::load(kv[u].e[e]), d4[(u * V + e) & 3]);
            const float dot = (d4[0] + d4[1]) + (d4[2] + d4[3]);
            sc = uniform ? 0.f : sh.scale * dot;
        }
        const float mnew = fmaxf(m, warp_max(sc));
        const float p = ok ? __expf(sc - mnew) : 0.f;
        const float corr = __expf(m - mnew);
        l = l * corr + warp_sum(p);
        m = mnew;
#pragma unroll
        for (int c = 0; c < CPL; c++) o[c] *= corr;
        const int nk = min(kWarpKeys, nvis - ch * kWarpKeys);
        __pipeline_wait_prior(0);
        __syncwarp();
        const T *vr = vs + lane * CPL;
#pragma unroll 8
        for (int jj = 0; jj < nk; jj++) {
            const float pj = __shfl_sync(0xffffffffu, p, jj);
            const T *vv = vr + (size_t)jj * DH;
            T vl[CPL];
            if constexpr (CPL * sizeof(T) == 16) {
                *reinterpret_cast<uint4 *>(vl) = *reinterpret_cast<const uint4 *>(vv);
            } else if constexpr (CPL * sizeof(T) == 8) {
                *reinterpret_cast<uint2 *>(vl) = *reinterpret_cast<const uint2 *>(vv);
            } else if constexpr (CPL * sizeof(T) == 4) {
                *reinterpret_cast<uint32_t *>(vl) = *reinterpret_cast<const uint32_t *>(vv);
            } else {
#pragma unroll
                for (int c = 0; c < CPL; c++) vl[c] = vv[c];
            }
#pragma unroll
            for (int c = 0; c < CPL; c++) o[c] = fmaf(pj, Elem<T>::load(vl[c]), o[c]);
        }
        __syncwarp();  // the warp's V buffer is refilled by the next chunk
    }
    // fold the NW warps
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
#pragma unroll
    for (int c = 0; c < CPL; c++) wo[warp][lane * CPL + c] = o[c];
    __syncthreads();
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w]);
    float Lsum = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w++) Lsum += wl[w] > 0.f ? wl[w] * __expf(wm[w] - M) : 0.f;
    // one column per thread (DH <= 256 threads); push the CTA's slice to CTA 0
    float oc = 0.f;
    if (threadIdx.x < DH) {
#pragma unroll
        for (int w = 0; w < NW; w++)
            if (wl[w] > 0.f) oc += wo[w][threadIdx.x] * __expf(wm[w] - M);
        cluster.map_shared_rank(&xo[0][0], 0)[rank * DH + threadIdx.x] = oc;
    }
    if (threadIdx.x == 0) {
        cluster.map_shared_rank(xm, 0)[rank] = M;
        cluster.map_shared_rank(xl, 0)[rank] = Lsum;
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x < DH) {
        float MM = -FLT_MAX;
        for (int r = 0; r < nsplit; r++) MM = fmaxf(MM, xm[r]);
        float LL = 0.f, OO = 0.f;
        for (int r = 0; r < nsplit; r++)
            if (xl[r] > 0.f) {
                const float w = __expf(xm[r] - MM);
                LL += xl[r] * w;
                OO += xo[r][threadIdx.x] * w;
            }
        stf(out, ((size_t)i * sh.nh + h) * DH + threadIdx.x, LL > 0.f ? OO / LL : 0.f);
    }
}

template <typename T, int DH, class Src, int NW>
int launch_warp_attn_nw(T *out, const T *q, Src src, const AttnShape &sh, int ns, cudaStream_t s, const void *pf_ptr,
                        size_t pf_bytes) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ns, (unsigned)(sh.S * sh.nh), 1);
    cfg.blockDim = dim3(NW * 32, 1, 1);
    cfg.dynamicSmemBytes = warp_attn_smem<T, DH, NW>();
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ns;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, attn_warp_kernel<T, DH, Src, NW>, q, src, out, sh, pf_ptr, pf_bytes);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "self_attention(warp): %s", cudaGetErrorString(e));
    return check_launch("self_attention(warp)");
}

template <typename T, int DH, class Src>
int launch_warp_attn(T *out, const T *q, Src src, const AttnShape &sh, cudaStream_t s, const void *pf_ptr,
                     size_t pf_bytes) {
    // slices: at most 3 chunks of 32 keys per CTA, so that a head's work is
    // spread over up to 8 SMs (the per-warp dot and P.V are latency-bound;
    // fewer busy warps per SM finish them sooner). CTAs of 4 warps (smaller,
    // to start beside the q/k/v projection) were measured slower.
    const int chunks = (sh.L + kWarpKeys - 1) / kWarpKeys;
    int ns = (chunks + 2) / 3;
    if (ns > kMaxCluster) ns = kMaxCluster;
    if (ns < 1) ns = 1;
    return launch_warp_attn_nw<T, DH, Src, 8>(out, q, src, sh, ns, s, pf_ptr, pf_bytes);
}

// ---- FAST prefill: query tiles on the tensor cores --------------------------
// One CTA = 64 consecutive query rows of one head (4 warps x 16 rows). K and V
// tiles of 64 keys stream through shared memory (cp.async, double-buffered,
// rows padded by 16 bytes so ldmatrix is free of bank conflicts). Each warp
// computes S = Q K^T for its 16 rows with mma.sync m16n8k16 (bf16/f16 in, f32
// accumulate), applies the causal mask (key j visible to query i when
// j <= i + L - S), folds the tile into a running max and sum (exp2 of scaled
// scores), and accumulates O += P V with P re-packed from the score
// registers as the A operand. Rows are normalised once at the end.
// Roofline at a 512-token prefill: tensor, 4*S*L*d*nh (causal: about half)
// flops; the K/V bytes are re-read from L2 by each query tile.
constexpr int kMQ = 64;       // query rows per CTA
constexpr int kMK = 64;       // keys per tile
constexpr int kMThreads = 128;

__device__ __forceinline__ uint32_t sm_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sm_u32(p)));
}
__device__ __forceinline__ void ldsm4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sm_u32(p)));
}
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&v);
    } else {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&v);
    }
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T, int DH> constexpr size_t mma_smem_bytes() {
    return (size_t)(kMQ + 4 * kMK) * (DH + 8) * sizeof(T);
}

template <typename T, int DH>
__global__ void __launch_bounds__(kMThreads) attn_mma_kernel(const T *__restrict__ q, KvDense<T> src,
                                                             T *__restrict__ out, AttnShape sh) {
    constexpr int RS = DH + 8;       // shared row stride (elements): 16-byte pad
    constexpr int CPR = DH / 8;      // 16-byte chunks per row
    constexpr int NKS = DH / 16;     // k-steps over the head dimension
    constexpr int NDT = DH / 8;      // 8-wide output column tiles
    extern __shared__ __align__(16) unsigned char smem[];
    T *qs = reinterpret_cast<T *>(smem);   // [kMQ][RS]
    T *ks = qs + kMQ * RS;                 // [2][kMK][RS]
    T *vs = ks + 2 * kMK * RS;             // [2][kMK][RS]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int q0 = blockIdx.x * kMQ, h = blockIdx.y;
    const int kvh = h * sh.nkvh / sh.nh;
    const int off = sh.L - sh.S;  // >= 0: the launcher sends L < S elsewhere
    const size_t kst = (size_t)sh.nkvh * DH;
    const T *kb = src.k + (size_t)kvh * DH, *vb = src.v + (size_t)kvh * DH;
    const int qn = min(kMQ, sh.S - q0);
    const int kend = min(sh.L, q0 + qn + off);  // keys [0, kend) are visible to some row of the tile
    const int ntiles = (kend + kMK - 1) / kMK;

    for (int c = tid; c < kMQ * CPR; c += kMThreads) {
        const int r = c / CPR, cc = c - r * CPR;
        T *dst = qs + r * RS + cc * 8;
        if (r < qn) __pipeline_memcpy_async(dst, q + ((size_t)(q0 + r) * sh.nh + h) * DH + cc * 8, 16);
        else *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
    }
    auto load_kv = [&](int tile) {
        if (tile < ntiles) {
            T *kd = ks + (tile & 1) * kMK * RS, *vd = vs + (tile & 1) * kMK * RS;
            for (int c = tid; c < kMK * CPR; c += kMThreads) {
                const int r = c / CPR, cc = c - r * CPR, j = tile * kMK + r;
                if (j < kend) {
                    __pipeline_memcpy_async(kd + r * RS + cc * 8, kb + (size_t)j * kst + cc * 8, 16);
                    __pipeline_memcpy_async(vd + r * RS + cc * 8, vb + (size_t)j * kst + cc * 8, 16);
                } else {
                    *reinterpret_cast<uint4 *>(kd + r * RS + cc * 8) = make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4 *>(vd + r * RS + cc * 8) = make_uint4(0, 0, 0, 0);
                }
            }
        }
        __pipeline_commit();
    };
    load_kv(0);  // one group: the Q tile and key tile 0
    load_kv(1);

    const float sc2 = sh.scale * 1.4426950408889634f;  // scores in log2 units
    const int qa = q0 + warp * 16 + g, qb = qa + 8;     // this thread's two query rows
    uint32_t qf[NKS][4];
    float o[NDT][4];
#pragma unroll
    for (int i = 0; i < NDT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

    for (int tile = 0; tile < ntiles; tile++) {
        __pipeline_wait_prior(1);
        __syncthreads();
        if (tile == 0) {
#pragma unroll
            for (int k = 0; k < NKS; k++)
                ldsm4(qf[k], qs + (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * RS + k * 16 + (lane >> 4) * 8);
        }
        const T *kt = ks + (tile & 1) * kMK * RS, *vt = vs + (tile & 1) * kMK * RS;
        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int k = 0; k < NKS; k++) {
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                uint32_t b[4];
                ldsm4(b, kt + (n * 8 + (lane & 7) + (lane >> 4) * 8) * RS + k * 16 + ((lane >> 3) & 1) * 8);
                mma16816<T>(s[n], qf[k], b[0], b[1]);
                mma16816<T>(s[n + 1], qf[k], b[2], b[3]);
            }
        }
        // scale, mask, running max per row (the 4 lanes of a quad share a row)
        const int j0 = tile * kMK;
        const bool edge = j0 + kMK > min(q0 + off + 1, kend);  // some key of this tile is masked for some row
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float v = s[n][c] * sc2;
                if (edge) {
                    const int j = j0 + n * 8 + 2 * t4 + (c & 1);
                    const int row = c < 2 ? qa : qb;
                    if (j >= kend || j > row + off) v = -INFINITY;
                }
                s[n][c] = v;
                mx[c >> 1] = fmaxf(mx[c >> 1], v);
            }
        }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mnew = fmaxf(mrow[r], mx[r]);
            corr[r] = mnew == -INFINITY ? 1.f : ex2(mrow[r] - mnew);
            mrow[r] = mnew;
            lrow[r] *= corr[r];
        }
#pragma unroll
        for (int i = 0; i < NDT; i++) {
            o[i][0] *= corr[0];
            o[i][1] *= corr[0];
            o[i][2] *= corr[1];
            o[i][3] *= corr[1];
        }
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float m = mrow[c >> 1];
                const float p = m == -INFINITY ? 0.f : ex2(s[n][c] - m);
                s[n][c] = p;
                lrow[c >> 1] += p;
            }
        }
        // O += P V: P (16 x 64) from the score registers, V via transposed ldmatrix
#pragma unroll
        for (int kk = 0; kk < kMK / 16; kk++) {
            uint32_t pa[4];
            pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int nd = 0; nd < NDT; nd += 2) {
                uint32_t b[4];
                ldsm4_t(b, vt + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * RS + nd * 8 + (lane >> 4) * 8);
                mma16816<T>(o[nd], pa, b[0], b[1]);
                mma16816<T>(o[nd + 1], pa, b[2], b[3]);
            }
        }
        __syncthreads();  // every warp is done with this buffer
        load_kv(tile + 2);
    }
    __pipeline_wait_prior(0);
    // row sums over the quad, then normalise and store
#pragma unroll
    for (int r = 0; r < 2; r++) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
    const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f, inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
#pragma unroll
    for (int nd = 0; nd < NDT; nd++) {
        const int col = nd * 8 + 2 * t4;
        if (qa < sh.S)
            *reinterpret_cast<uint32_t *>(out + ((size_t)qa * sh.nh + h) * DH + col) =
                pack2<T>(o[nd][0] * inv0, o[nd][1] * inv0);
        if (qb < sh.S)
            *reinterpret_cast<uint32_t *>(out + ((size_t)qb * sh.nh + h) * DH + col) =
                pack2<T>(o[nd][2] * inv1, o[nd][3] * inv1);
    }
}

template <typename T, int DH>
int launch_mma_attn(T *out, const T *q, KvDense<T> src, const AttnShape &sh, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((sh.S + kMQ - 1) / kMQ), (unsigned)sh.nh, 1);
    cfg.blockDim = dim3(kMThreads, 1, 1);
    cfg.dynamicSmemBytes = mma_smem_bytes<T, DH>();
    cfg.stream = s;
    cfg.numAttrs = 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, attn_mma_kernel<T, DH>, q, src, out, sh);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "self_attention(mma): %s", cudaGetErrorString(e));
    return check_launch("self_attention(mma)");
}

// ---- FAST batched decode: GQA groups on the tensor cores, K/V by TMA --------
// One CTA = one (sequence, kv head) and one slice of its keys. The hpc query
// heads that share the kv head are the 16 rows of an m16n8k16 A tile (rows
// past hpc are zero), so every K/V row is read once per kv head and feeds
// hpc query heads through mma.sync. A producer warp streams the slice in
// stages of kDStage keys: one TMA box of K and one of V per stage (the kv
// head's DH columns as DH/64 blocks of 128 bytes, 128-byte swizzle; 16 KB
// per box at DH = 128) into a ring of kDS stages on full/empty mbarriers.
// Four consumer warps take 16 keys of each stage, keep a running max/sum per
// row and O += P V in registers. Few large boxes keep about 200 KB in flight
// per SM (two CTAs), enough to stream at HBM rate; per-warp cp.async tiles of
// 16 keys left the kernel waiting on its loads at 0.47 of HBM. After the key
// loop the ring holds the warps' partial rows, the warps fold in shared
// memory, then the CTAs of the cluster (the key slices) fold in CTA 0 through
// distributed shared memory.
// Roofline: HBM, 2 * B * L * nkvh * d * size bytes of K/V.
constexpr int kDW = 4;                     // consumer warps per CTA
constexpr int kDThreads = (kDW + 1) * 32;  // and the producer warp
constexpr int kDK = 16;                    // keys per consumer warp and stage
constexpr int kDN = kDK / 8;               // n-tiles of 8 keys
constexpr int kDStage = kDW * kDK;         // keys per stage
constexpr int kDS = 3;                     // ring stages
constexpr long long kDWaitCycles = 2000000000ll;  // ~1 s: a wait that long records an error

template <typename T, int DH> struct MmaDecLayout {
    static constexpr int RS = DH + 8;                                // Q tile row stride (elements)
    static constexpr size_t box = (size_t)kDStage * DH * sizeof(T);  // one K or V box
    static constexpr size_t stage = 2 * box;
    static constexpr size_t qs = kDS * stage;  // [16][RS] T after the ring (ring at 0, 1024-aligned)
    // + 1 KB: the ring starts at the first 1024-byte boundary of dynamic
    // shared memory (TMA boxes with 128-byte swizzle)
    static constexpr size_t bytes = qs + (size_t)16 * RS * sizeof(T) + 1024;
    // reused from the ring after the key loop: each consumer warp's
    // unnormalised [16][DH] f32 rows, then (CTA 0) the slices' [ns][hpc][DH]
    static constexpr size_t xo = (size_t)kDW * 16 * DH * 4;
    static_assert(xo + (size_t)kMaxCluster * 16 * DH * 4 <= qs, "the fold areas must fit in the ring");
};

// Byte offset of 16-byte chunk ch (of DH / 8) of box row r: the box is DH / 64
// blocks of [kDStage rows][128 bytes], chunk c of row r stored at c ^ (r % 8).
__device__ __forceinline__ uint32_t dec_swz(int r, int ch) {
    return (uint32_t)((ch >> 3) * (kDStage * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}
__device__ __forceinline__ void ldsm4a(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm4a_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

template <typename T, int DH>
__global__ void __launch_bounds__(kDThreads) attn_mma_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                    const __grid_constant__ CUtensorMap tmV,
                                                                    const T *__restrict__ q, KvCache<T> src,
                                                                    T *__restrict__ out, AttnShape sh,
                                                                    int rows_per_seq, unsigned long long *err) {
    using Lay = MmaDecLayout<T, DH>;
    constexpr int RS = Lay::RS, CPR = DH / 8, NKS = DH / 16, NDT = DH / 8;
    // the dynamic shared memory symbol is shared with this file's other
    // kernels (16-byte alignment): the ring's 1024-byte boundary is found at
    // run time, the same offset in every CTA of the cluster
    extern __shared__ __align__(16) unsigned char smem_raw_dec[];
    unsigned char *smem = smem_raw_dec + ((1024u - (smem_u32(smem_raw_dec) & 1023u)) & 1023u);
    T *qs = reinterpret_cast<T *>(smem + Lay::qs);
    __shared__ __align__(8) uint64_t full[kDS], empty[kDS];
    __shared__ float wm[kDW][16], wl[kDW][16];
    __shared__ float xm[kMaxCluster][16], xl[kMaxCluster][16];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank(), ns = (int)cluster.num_blocks();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int b = blockIdx.y / sh.nkvh, kvh = blockIdx.y % sh.nkvh;
    const int hpc = sh.nh / sh.nkvh, h0 = kvh * hpc;
    const T *k, *v;
    int nkeys, nvis;
    bool uniform;
    src.row(sh, b, k, v, nkeys, nvis, uniform);  // lengths were set by an earlier step
    const int per = (nvis + ns - 1) / ns;
    const int c0 = min(rank * per, nvis), c1 = min(c0 + per, nvis);
    const int nst = (c1 - c0 + kDStage - 1) / kDStage;  // stages of this slice
    if (tid == 0) {
        for (int s = 0; s < kDS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kDW);
        }
        mbar_init_fence();
    }
    __syncthreads();
    pdl_trigger();
    const float sc2 = sh.scale * 1.4426950408889634f;
    float o[NDT][4];
#pragma unroll
    for (int i = 0; i < NDT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

    if (warp == kDW) {
        // producer: stage t holds keys [c0 + t kDStage, c0 + (t + 1) kDStage);
        // rows past c1 are masked (K) or cleared (V) by the consumers. Rows
        // before the newest one were written by earlier steps, so they are
        // requested before the wait for the previous kernel.
        if (lane == 0) {
            const int row0 = b * rows_per_seq + c0, blk = kvh * (DH / 64);
            bool waited = false;
            for (int t = 0; t < nst; t++) {
                const int s = t % kDS;
                if (t >= kDS && !mbar_wait(&empty[s], ((t / kDS) - 1) & 1, kDWaitCycles)) {
                    record_device_error(err, 9, (long long)blockIdx.y);
                    break;
                }
                if (!waited && c0 + (t + 1) * kDStage >= nvis) {
                    pdl_wait();  // this stage holds the newest row
                    waited = true;
                }
                unsigned char *st = smem + (size_t)s * Lay::stage;
                mbar_arrive_expect_tx(&full[s], (unsigned)Lay::stage);
                tma_load_box3(st, &tmK, 0, row0 + t * kDStage, blk, &full[s]);
                tma_load_box3(st + Lay::box, &tmV, 0, row0 + t * kDStage, blk, &full[s]);
            }
        }
    } else {
        pdl_wait();  // q comes from the previous kernel
        for (int c = tid; c < 16 * CPR; c += kDW * 32) {
            const int r = c / CPR, cc = c - r * CPR;
            T *dst = qs + r * RS + cc * 8;
            if (r < hpc) __pipeline_memcpy_async(dst, q + ((size_t)b * sh.nh + h0 + r) * DH + cc * 8, 16);
            else *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
        }
        __pipeline_commit();
        __pipeline_wait_prior(0);
        asm volatile("bar.sync 1, %0;" ::"r"(kDW * 32) : "memory");  // the Q tile is shared by the consumers
        uint32_t qf[NKS][4];
#pragma unroll
        for (int kk = 0; kk < NKS; kk++)
            ldsm4(qf[kk], qs + ((lane & 7) + ((lane >> 3) & 1) * 8) * RS + kk * 16 + (lane >> 4) * 8);
        bool bad = false;
        const int wr = warp * kDK;  // this warp's first row of each stage
        for (int t = 0; t < nst; t++) {
            const int s = t % kDS;
            if (!bad && !mbar_wait(&full[s], (t / kDS) & 1, kDWaitCycles)) {
                if (lane == 0) record_device_error(err, 9, (long long)blockIdx.y);
                bad = true;
            }
            const int j0 = c0 + t * kDStage + wr;  // key of this warp's first row
            const uint32_t kt = smem_u32(smem + (size_t)s * Lay::stage), vt = kt + (uint32_t)Lay::box;
            if (!bad && j0 < c1) {
                if (j0 + kDK > c1) {
                    // rows past the slice hold other positions (or fill):
                    // their V rows are cleared so that P = 0 meets finite values
                    for (int e = lane; e < kDK * CPR; e += 32) {
                        const int r = e / CPR, ch = e - r * CPR;
                        if (j0 + r >= c1) {
                            const uint32_t a = vt + dec_swz(wr + r, ch);
                            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
                        }
                    }
                    // written through the generic proxy: ordered before the
                    // next TMA into this stage
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                }
                float sacc[kDN][4];
#pragma unroll
                for (int n = 0; n < kDN; n++) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < NKS; kk++) {
#pragma unroll
                    for (int n = 0; n < kDN; n += 2) {
                        uint32_t bb[4];
                        ldsm4a(bb, kt + dec_swz(wr + n * 8 + (lane & 7) + (lane >> 4) * 8, kk * 2 + ((lane >> 3) & 1)));
                        mma16816<T>(sacc[n], qf[kk], bb[0], bb[1]);
                        mma16816<T>(sacc[n + 1], qf[kk], bb[2], bb[3]);
                    }
                }
                float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
                for (int n = 0; n < kDN; n++) {
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const int j = j0 + n * 8 + 2 * t4 + (c & 1);
                        const float val = j < c1 ? sacc[n][c] * sc2 : -INFINITY;
                        sacc[n][c] = val;
                        mx[c >> 1] = fmaxf(mx[c >> 1], val);
                    }
                }
                float corr[2];
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                    const float mnew = fmaxf(mrow[r], mx[r]);
                    corr[r] = mnew == -INFINITY ? 1.f : ex2(mrow[r] - mnew);
                    mrow[r] = mnew;
                    lrow[r] *= corr[r];
                }
#pragma unroll
                for (int i = 0; i < NDT; i++) {
                    o[i][0] *= corr[0];
                    o[i][1] *= corr[0];
                    o[i][2] *= corr[1];
                    o[i][3] *= corr[1];
                }
#pragma unroll
                for (int n = 0; n < kDN; n++) {
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const float m = mrow[c >> 1];
                        const float p = m == -INFINITY ? 0.f : ex2(sacc[n][c] - m);
                        sacc[n][c] = p;
                        lrow[c >> 1] += p;
                    }
                }
                uint32_t pa[4];
                pa[0] = pack2<T>(sacc[0][0], sacc[0][1]);
                pa[1] = pack2<T>(sacc[0][2], sacc[0][3]);
                pa[2] = pack2<T>(sacc[1][0], sacc[1][1]);
                pa[3] = pack2<T>(sacc[1][2], sacc[1][3]);
#pragma unroll
                for (int nd = 0; nd < NDT; nd += 2) {
                    uint32_t bb[4];
                    ldsm4a_t(bb, vt + dec_swz(wr + (lane & 7) + ((lane >> 3) & 1) * 8, nd + (lane >> 4)));
                    mma16816<T>(o[nd], pa, bb[0], bb[1]);
                    mma16816<T>(o[nd + 1], pa, bb[2], bb[3]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
#pragma unroll
        for (int r = 0; r < 2; r++) {
            lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
            lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
        }
        if (t4 == 0) {
            wm[warp][g] = mrow[0];
            wm[warp][g + 8] = mrow[1];
            wl[warp][g] = lrow[0];
            wl[warp][g + 8] = lrow[1];
        }
        // every consumer is past its last stage (and so every box has landed):
        // this warp's unnormalised rows, [16][DH] f32, go into the ring
        asm volatile("bar.sync 1, %0;" ::"r"(kDW * 32) : "memory");
        float *ow = reinterpret_cast<float *>(smem) + (size_t)warp * 16 * DH;
#pragma unroll
        for (int nd = 0; nd < NDT; nd++) {
            const int col = nd * 8 + 2 * t4;
            ow[g * DH + col] = o[nd][0];
            ow[g * DH + col + 1] = o[nd][1];
            ow[(g + 8) * DH + col] = o[nd][2];
            ow[(g + 8) * DH + col + 1] = o[nd][3];
        }
    }
    __syncthreads();
    cluster.sync();  // every CTA is past its key loop: CTA 0's ring may take the slices' rows
    // fold the warps into this CTA's slice and push it to CTA 0 of the cluster
    float *xo0 = cluster.map_shared_rank(reinterpret_cast<float *>(smem + Lay::xo), 0);
    float *xm0 = cluster.map_shared_rank(&xm[0][0], 0), *xl0 = cluster.map_shared_rank(&xl[0][0], 0);
    for (int x = tid; x < hpc * DH; x += kDThreads) {
        const int row = x / DH, col = x - row * DH;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDW; w++) M = fmaxf(M, wm[w][row]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kDW; w++) {
                if (wl[w][row] > 0.f) {
                    const float e = ex2(wm[w][row] - M);
                    L += wl[w][row] * e;
                    O += reinterpret_cast<const float *>(smem)[((size_t)w * 16 + row) * DH + col] * e;
                }
            }
        }
        xo0[((size_t)rank * hpc + row) * DH + col] = O;
        if (col == 0) {
            xm0[rank * 16 + row] = M;
            xl0[rank * 16 + row] = L;
        }
    }
    cluster.sync();
    if (rank == 0) {
        const float *xo = reinterpret_cast<const float *>(smem + Lay::xo);
        for (int x = tid; x < hpc * DH; x += kDThreads) {
            const int row = x / DH, col = x - row * DH;
            float MM = -INFINITY;
            for (int r = 0; r < ns; r++) MM = fmaxf(MM, xm[r][row]);
            float LL = 0.f, OO = 0.f;
            if (MM != -INFINITY) {
                for (int r = 0; r < ns; r++) {
                    if (xl[r][row] > 0.f) {
                        const float e = ex2(xm[r][row] - MM);
                        LL += xl[r][row] * e;
                        OO += xo[((size_t)r * hpc + row) * DH + col] * e;
                    }
                }
            }
            stf(out, ((size_t)b * sh.nh + h0 + row) * DH + col, LL > 0.f ? OO / LL : 0.f);
        }
    }
}

// Slices per (sequence, kv head): as many as keep every CTA of the launch
// resident at once (two per SM), at least 128 keys per slice, at most a
// portable cluster. One wave of long slices beats several waves of short
// ones: at 64 sequences x 2 kv heads x 2300 keys, 2 slices (256 CTAs) ran
// the step's attention in 36 us serialised, 5 slices (640 CTAs) in 45 us,
// 8 in 53 us. Depends only on the batch and the cache capacity, so a captured
// graph stays valid as the caches grow.
inline int mma_decode_slices(const AttnShape &sh) {
    const long pairs = (long)sh.S * sh.nkvh;
    long ns = 2L * sm_count() / (pairs > 0 ? pairs : 1);
    const long by_len = sh.L / 128;
    if (ns > by_len) ns = by_len;
    if (ns > kMaxCluster) ns = kMaxCluster;
    if (ns < 1) ns = 1;
    return (int)ns;
}

// The TMA view of a cache: [B * rows_per_seq rows][nkvh * d columns]; false
// when the caches do not have that shape or the driver refuses the maps.
template <typename T>
bool mma_decode_maps(CUtensorMap *tk, CUtensorMap *tv, const KvCache<T> &src, const AttnShape &sh, int &rows_per_seq) {
    const size_t w = (size_t)sh.nkvh * sh.d;
    if (src.seq_stride % w || !aligned16(src.k) || !aligned16(src.v)) return false;
    const size_t rps = src.seq_stride / w, rows = (size_t)sh.S * rps;
    if (rps < (size_t)sh.L || rows >= (1ull << 31) || w >= (1ull << 31)) return false;
    rows_per_seq = (int)rps;
    return tma_map_row_stages(tk, src.k, (int)sizeof(T), (int)rows, (int)w, kDStage, sh.d / 64) &&
           tma_map_row_stages(tv, src.v, (int)sizeof(T), (int)rows, (int)w, kDStage, sh.d / 64);
}

template <typename T, int DH>
int launch_mma_decode(T *out, const T *q, KvCache<T> src, const AttnShape &sh, const CUtensorMap &tk,
                      const CUtensorMap &tv, int rows_per_seq, cudaStream_t s) {
    const int ns = mma_decode_slices(sh);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ns, (unsigned)(sh.S * sh.nkvh), 1);
    cfg.blockDim = dim3(kDThreads, 1, 1);
    cfg.dynamicSmemBytes = MmaDecLayout<T, DH>::bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ns;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e =
        cudaLaunchKernelEx(&cfg, attn_mma_decode_kernel<T, DH>, tk, tv, q, src, out, sh, rows_per_seq, dev_error_ptr());
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "self_attention(mma decode): %s", cudaGetErrorString(e));
    return check_launch("self_attention(mma decode)");
}

// ---- REFERENCE order --------------------------------------------------------
template <typename T, class Src, bool kVec>
__global__ void __launch_bounds__(kThreads) attn_ref_kernel(const T *__restrict__ q, Src src, T *__restrict__ out,
                                                            float *__restrict__ gscores, AttnShape sh) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float s_red[kThreads / 32];
    __shared__ float s_max, s_sum;
    constexpr int es = sizeof(T);
    const int i = blockIdx.x / sh.nh, h = blockIdx.x % sh.nh;
    const int kvh = h * sh.nkvh / sh.nh;
    const int wmax = sh.d > sh.dv ? sh.d : sh.dv;
    const int rst = pad_row(wmax, es);  // shared row stride (elements)
    float *qs = reinterpret_cast<float *>(smem);
    T *tile = reinterpret_cast<T *>(smem + ((sh.d * 4 + 15) & ~15));
    float *sc = gscores ? gscores + (size_t)blockIdx.x * sh.L
                        : reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(tile) + (size_t)kRefChunk * rst * es);
    const int tid = threadIdx.x;
    const T *k, *v;
    int nkeys, nvis;
    bool uniform;
    src.row(sh, i, k, v, nkeys, nvis, uniform);
    const size_t kstride = (size_t)sh.nkvh * sh.d, vstride = (size_t)sh.nkvh * sh.dv;
    const T *kb = k + (size_t)kvh * sh.d, *vb = v + (size_t)kvh * sh.dv;
    for (int c = tid; c < sh.d; c += kThreads) qs[c] = ldf(q, ((size_t)i * sh.nh + h) * sh.d + c);
    // masked / uniform keys first (no dot product needed)
    for (int j = tid; j < nkeys; j += kThreads)
        if (uniform || j >= nvis) sc[j] = -1e9f;
    // scores: sequential dot, then scale * dot (self_attention_cpu.cpp:37-45)
    const int nscore = uniform ? 0 : nvis;
    for (int c0 = 0; c0 < nscore; c0 += kRefChunk) {
        const int nc = min(kRefChunk, nscore - c0);
        __syncthreads();
        load_tile<T, kVec>(tile, kb + (size_t)c0 * kstride, nc, sh.d, kstride, rst);
        __pipeline_commit();
        __pipeline_wait_prior(0);
        __syncthreads();
        if (tid < nc) {
            const T *kr = tile + (size_t)tid * rst;
            float a = 0.f;
            for (int c = 0; c < sh.d; c++) a = __fadd_rn(a, __fmul_rn(qs[c], Elem<T>::load(kr[c])));
            sc[c0 + tid] = __fmul_rn(sh.scale, a);
        }
    }
    __syncthreads();
    float mx = -FLT_MAX;
    for (int j = tid; j < nkeys; j += kThreads) mx = fmaxf(mx, sc[j]);
    mx = warp_max(mx);
    if ((tid & 31) == 0) s_red[tid >> 5] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = s_red[0];
        for (int w = 1; w < kThreads / 32; w++) m = fmaxf(m, s_red[w]);
        s_max = m;
    }
    __syncthreads();
    mx = s_max;
    for (int j = tid; j < nkeys; j += kThreads) sc[j] = expf_glibc(__fsub_rn(sc[j], mx));
    __syncthreads();
    if (tid == 0) {  // sequential sum over every key (self_attention_cpu.cpp:70-74)
        float sum = 0.f;
        for (int j = 0; j < nkeys; j++) sum = __fadd_rn(sum, sc[j]);
        s_sum = sum;
    }
    __syncthreads();
    const float sum = s_sum;
    for (int j = tid; j < nkeys; j += kThreads) sc[j] = __fdiv_rn(sc[j], sum);
    // output: sequential sum over keys of round(p * v). Masked keys carry
    // exact zeros and leave the sum unchanged, so the chain stops at nvis.
    float a[4] = {0.f, 0.f, 0.f, 0.f};  // columns tid, tid+256, ... (dv <= 1024)
    for (int c0 = 0; c0 < nvis; c0 += kRefChunk) {
        const int nc = min(kRefChunk, nvis - c0);
        __syncthreads();
        load_tile<T, kVec>(tile, vb + (size_t)c0 * vstride, nc, sh.dv, vstride, rst);
        __pipeline_commit();
        __pipeline_wait_prior(0);
        __syncthreads();
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int c = tid + u * kThreads;
            if (c < sh.dv) {
                float acc = a[u];
                for (int jj = 0; jj < nc; jj++)
                    acc = __fadd_rn(acc, __fmul_rn(sc[c0 + jj], Elem<T>::load(tile[(size_t)jj * rst + c])));
                a[u] = acc;
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int c = tid + u * kThreads;
        if (c < sh.dv) stf(out, ((size_t)i * sh.nh + h) * sh.dv + c, a[u]);
    }
}

size_t ref_smem_bytes(const AttnShape &sh, int es, bool global_scores) {
    const int wmax = sh.d > sh.dv ? sh.d : sh.dv;
    size_t b = (size_t)((sh.d * 4 + 15) & ~15) + (size_t)kRefChunk * pad_row(wmax, es) * es;
    if (!global_scores) b += (size_t)sh.L * 4;
    return b;
}

// Heads per CTA: all heads of a kv group (up to 8) share each K/V tile when
// there are enough query rows to fill the GPU; with few rows (decode) one
// head per CTA gives 6x more CTAs and keeps each CTA's serial work short.
int pick_hpc(int G, int dv, long rows_x_heads) {
    if (rows_x_heads < 2L * sm_count()) return 1;
    for (int h = (G < 8 ? G : 8); h >= 1; h--)
        if (G % h == 0 && h * dv <= kMaxAcc * kThreads) return h;
    return 1;
}

AttnShape make_shape(size_t S, size_t nh, size_t nkvh, size_t d, size_t dv, size_t L, float scale) {
    AttnShape sh{};
    sh.S = (int)S;
    sh.nh = (int)nh;
    sh.nkvh = (int)nkvh;
    sh.d = (int)d;
    sh.dv = (int)dv;
    sh.L = (int)L;
    sh.scale = scale;
    sh.hpc = pick_hpc((int)(nh / nkvh), (int)dv, (long)S * (long)nh);
    const long rows = (long)S * (long)(nh / sh.hpc);
    const long target = 2L * sm_count();
    long ns = rows >= target ? 1 : (target + rows - 1) / rows;
    const long tiles = ((long)L + kKT - 1) / kKT;
    if (ns > tiles) ns = tiles;
    if (ns > kMaxCluster) ns = kMaxCluster;
    sh.nsplit = (int)(ns < 1 ? 1 : ns);
    return sh;
}

// FAST needs no workspace (the cluster folds its slices in shared memory);
// REFERENCE keeps one score per key in global memory when the cache is too
// long for shared memory.
size_t ws_bytes(const AttnShape &sh, bool ref) {
    if (ref) return sh.L > kRefSmemScores ? (size_t)sh.S * sh.nh * sh.L * sizeof(float) : 0;
    return 0;
}

// Raises the dynamic shared-memory limits once per device (a non-stream call,
// kept out of graph capture).
template <typename T, class Src> void set_attrs() {
    const int lim = 200 * 1024;
    cudaFuncSetAttribute(attn_ref_kernel<T, Src, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(attn_ref_kernel<T, Src, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(attn_fast_kernel<T, Src, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(attn_fast_kernel<T, Src, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if constexpr (sizeof(T) == 2 && IsKvCache<Src>::value) {
        cudaFuncSetAttribute(attn_mma_decode_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)MmaDecLayout<T, 128>::bytes);
        cudaFuncSetAttribute(attn_mma_decode_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)MmaDecLayout<T, 64>::bytes);
    }
    if constexpr (sizeof(T) == 2) {
        cudaFuncSetAttribute(attn_mma_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)mma_smem_bytes<T, 128>());
        cudaFuncSetAttribute(attn_mma_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)mma_smem_bytes<T, 64>());
    }
    cudaFuncSetAttribute(attn_warp_kernel<T, 128, Src, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)warp_attn_smem<T, 128, 8>());
    cudaFuncSetAttribute(attn_warp_kernel<T, 64, Src, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)warp_attn_smem<T, 64, 8>());
}

void init_attrs_once() {
    static thread_local unsigned long long done_mask = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || (done_mask >> dev) & 1ull) return;
    set_attrs<float, KvDense<float>>();
    set_attrs<__nv_bfloat16, KvDense<__nv_bfloat16>>();
    set_attrs<__half, KvDense<__half>>();
    set_attrs<float, KvCache<float>>();
    set_attrs<__nv_bfloat16, KvCache<__nv_bfloat16>>();
    set_attrs<__half, KvCache<__half>>();
    done_mask |= 1ull << dev;
}

template <typename T> bool vec_ok(const AttnShape &sh, const void *k, const void *v, size_t kstride_bytes_extra = 0) {
    const int es = sizeof(T);
    return ((sh.d * es) % 16 == 0) && ((sh.dv * es) % 16 == 0) && aligned16(k) && aligned16(v) &&
           ((size_t)sh.nkvh * sh.d * es) % 16 == 0 && ((size_t)sh.nkvh * sh.dv * es) % 16 == 0 &&
           kstride_bytes_extra % 16 == 0;
}

template <typename T, class Src>
int launch_attn(T *out, const T *q, Src src, const AttnShape &sh, bool ref, void *ws, cudaStream_t s, bool vec,
                const void *pf_ptr = nullptr, size_t pf_bytes = 0) {
    init_attrs_once();
    if (ref) {
        const bool g = sh.L > kRefSmemScores;
        const size_t smem = ref_smem_bytes(sh, sizeof(T), g);
        if (vec) attn_ref_kernel<T, Src, true><<<sh.S * sh.nh, kThreads, smem, s>>>(q, src, out, g ? (float *)ws : nullptr, sh);
        else attn_ref_kernel<T, Src, false><<<sh.S * sh.nh, kThreads, smem, s>>>(q, src, out, g ? (float *)ws : nullptr, sh);
        return check_launch("self_attention(reference)");
    }
    if constexpr (sizeof(T) == 2 && IsKvCache<Src>::value) {
        // batched decode: one CTA per (sequence, kv head) and key slice, the
        // query heads of the group as the rows of a tensor-core tile
        CUtensorMap tk, tv;
        int rps = 0;
        if (vec && sh.d == sh.dv && (sh.d == 128 || sh.d == 64) && sh.nh / sh.nkvh <= 16 && sh.S * sh.nkvh >= 32 &&
            mma_decode_maps(&tk, &tv, src, sh, rps))
            return sh.d == 128 ? launch_mma_decode<T, 128>(out, q, src, sh, tk, tv, rps, s)
                               : launch_mma_decode<T, 64>(out, q, src, sh, tk, tv, rps, s);
    }
    if (vec && sh.d == sh.dv && (sh.d == 128 || sh.d == 64) && (long)sh.S * sh.nh < 2L * sm_count()) {
        // few query rows: one head per warp-group, no block barriers in the key loop
        return sh.d == 128 ? launch_warp_attn<T, 128, Src>(out, q, src, sh, s, pf_ptr, pf_bytes)
                           : launch_warp_attn<T, 64, Src>(out, q, src, sh, s, pf_ptr, pf_bytes);
    }
    if constexpr (sizeof(T) == 2 && !IsKvCache<Src>::value) {
        if (vec && sh.d == sh.dv && (sh.d == 128 || sh.d == 64) && sh.L >= sh.S)
            return sh.d == 128 ? launch_mma_attn<T, 128>(out, q, src, sh, s)
                               : launch_mma_attn<T, 64>(out, q, src, sh, s);
    }
    const FastSmem lay = fast_smem(sh, sizeof(T));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sh.nsplit, (unsigned)(sh.S * (sh.nh / sh.hpc)), 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)lay.bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)sh.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e = vec ? cudaLaunchKernelEx(&cfg, attn_fast_kernel<T, Src, true>, q, src, out, sh)
                        : cudaLaunchKernelEx(&cfg, attn_fast_kernel<T, Src, false>, q, src, out, sh);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "self_attention(fast): %s", cudaGetErrorString(e));
    return check_launch("self_attention(fast)");
}

// Library-owned workspace for the allocation-free-signature entry point.
struct Workspace {
    void *p = nullptr;
    size_t bytes = 0;
};
thread_local Workspace t_ws[64];

int check_args(const void *o, const void *q, const void *k, const void *v, size_t S, size_t nh, size_t nkvh, size_t d,
               size_t dv, size_t L, wginferDataType_t dtype) {
    WGB_REQUIRE(o && q && k && v, WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: null pointer");
    WGB_REQUIRE(nkvh > 0 && nh % nkvh == 0, WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: nhead %% nkvhead != 0");
    const size_t es = dtype == WGINFER_DTYPE_F32 ? 4 : 2;
    // two double-buffered K/V tiles of kKT keys must fit in shared memory
    WGB_REQUIRE(d > 0 && dv > 0 && (d + dv) * es <= 1024, WGB_ERR_INVALID_ARGUMENT,
                "wgb_self_attention: (d + dv) * element size must be <= 1024 bytes (d=%zu, dv=%zu)", d, dv);
    WGB_REQUIRE(S < (1u << 20) && L < (1u << 30) && nh < 4096, WGB_ERR_INVALID_ARGUMENT,
                "wgb_self_attention: size too large");
    WGB_REQUIRE(S * nh < 65536u,
                WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: too many query rows x heads");
    return WGB_OK;
}

}  // namespace

void attn_prepare() { init_attrs_once(); }

size_t attn_decode_workspace(int B, int nh, int nkvh, int dh, int maxlen, bool ref) {
    AttnShape sh = make_shape((size_t)B, (size_t)nh, (size_t)nkvh, (size_t)dh, (size_t)dh, (size_t)maxlen, 1.f);
    return ws_bytes(sh, ref);
}

int attn_decode(wginferDataType_t dtype, void *out, const void *q, const void *kcache, const void *vcache,
                size_t seq_stride, const int64_t *lens, int B, int nh, int nkvh, int dh, int maxlen, float scale,
                void *ws, bool ref, cudaStream_t s, const void *pf_ptr, size_t pf_bytes) {
    // The cluster size depends only on maxlen, so a captured graph stays valid
    // as the sequences grow; each row splits its own visible keys.
    AttnShape sh = make_shape((size_t)B, (size_t)nh, (size_t)nkvh, (size_t)dh, (size_t)dh, (size_t)maxlen, scale);
    WGB_DISPATCH_FLOAT(dtype, T,
        const bool vec = vec_ok<T>(sh, kcache, vcache, seq_stride * sizeof(T));
        return launch_attn((T *)out, (const T *)q,
                           KvCache<T>{(const T *)kcache, (const T *)vcache, seq_stride, lens}, sh, ref, ws, s, vec,
                           pf_ptr, pf_bytes));
    return WGB_OK;
}

}  // namespace wgb

extern "C" size_t wgb_self_attention_workspace_size(size_t seqlen, size_t nhead, size_t nkvhead, size_t d, size_t dv,
                                                    size_t total_len) {
    if (seqlen == 0 || total_len == 0 || nkvhead == 0 || nhead % nkvhead) return 0;
    wgb::AttnShape sh = wgb::make_shape(seqlen, nhead, nkvhead, d, dv, total_len, 1.f);
    return wgb::ws_bytes(sh, wgb::current_numerics() == WGB_NUMERICS_REFERENCE);
}

extern "C" int wgb_self_attention_ex(void *attn_val, const void *q, const void *k, const void *v,
                                     wginferDataType_t dtype, size_t seqlen, size_t nhead, size_t nkvhead, size_t d,
                                     size_t dv, size_t total_len, float scale, void *workspace, size_t workspace_bytes,
                                     wginferStream_t stream) {
    if (seqlen == 0 || nhead == 0) return WGB_OK;
    int rc = wgb::check_args(attn_val, q, k, v, seqlen, nhead, nkvhead, d, dv, total_len, dtype);
    if (rc) return rc;
    if (total_len == 0) return wgb::set_error(WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: total_len == 0");
    const bool ref = wgb::current_numerics() == WGB_NUMERICS_REFERENCE;
    wgb::AttnShape sh = wgb::make_shape(seqlen, nhead, nkvhead, d, dv, total_len, scale);
    const size_t need = wgb::ws_bytes(sh, ref);
    WGB_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr), WGB_ERR_INVALID_ARGUMENT,
                "wgb_self_attention_ex: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    WGB_DISPATCH_FLOAT(dtype, T,
        const bool vec = wgb::vec_ok<T>(sh, k, v);
        return wgb::launch_attn((T *)attn_val, (const T *)q, wgb::KvDense<T>{(const T *)k, (const T *)v}, sh, ref,
                                workspace, (cudaStream_t)stream, vec));
    return WGB_OK;
}

extern "C" int wgb_self_attention(void *attn_val, const void *q, const void *k, const void *v, wginferDataType_t dtype,
                                  size_t seqlen, size_t nhead, size_t nkvhead, size_t d, size_t dv, size_t total_len,
                                  float scale, wginferStream_t stream) {
    if (seqlen == 0 || nhead == 0) return WGB_OK;
    int rc = wgb::check_args(attn_val, q, k, v, seqlen, nhead, nkvhead, d, dv, total_len, dtype);
    if (rc) return rc;
    const size_t need = wgb_self_attention_workspace_size(seqlen, nhead, nkvhead, d, dv, total_len);
    void *ws = nullptr;
    if (need) {
        int dev = 0;
        cudaGetDevice(&dev);
        WGB_REQUIRE(dev >= 0 && dev < 64, WGB_ERR_INVALID_ARGUMENT, "device id %d", dev);
        wgb::Workspace &w = wgb::t_ws[dev];
        if (w.bytes < need) {
            // the old buffer may still be in use by work queued on `stream`
            if (w.p) {
                cudaStreamSynchronize((cudaStream_t)stream);
                cudaFree(w.p);
            }
            w.p = nullptr;
            w.bytes = 0;
            if (cudaMalloc(&w.p, need) != cudaSuccess) {
                cudaGetLastError();
                return wgb::set_error(WGB_ERR_NO_MEMORY, "wgb_self_attention: workspace of %zu bytes", need);
            }
            w.bytes = need;
        }
        ws = w.p;
    }
    return wgb_self_attention_ex(attn_val, q, k, v, dtype, seqlen, nhead, nkvhead, d, dv, total_len, scale, ws, need,
                                 stream);
}

// ---- allocation-free variant -------------------------------------------------
// Some callers cannot call cudaMalloc: code running inside an allocator or
// memory-pool callback (re-entering the allocator would deadlock), host
// runtimes that own every byte of device memory and give their kernels no
// allocation hook, and real-time threads that must not block in the driver.
// wgb_self_attention_noalloc serves them with a fixed scratch array compiled
// into this library instead of the lazily allocated workspace.
namespace wgb {
namespace {

constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB, held by every GPU that loads the library
static __device__ __align__(256) unsigned char g_attn_static_scratch[kStaticScratchBytes];

// The array's name in host code is only a host-side stand-in; its device
// address is looked up on every call, with the caller's device current (the
// lookup is cheap, and an address kept from an earlier call would be stale
// after a cudaDeviceReset reloads the module).
int static_scratch(void **out) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
    if (e != cudaSuccess || p == nullptr)
        return set_error(WGB_ERR_CUDA, "wgb_self_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    *out = p;
    return WGB_OK;
}

}  // namespace
}  // namespace wgb

extern "C" size_t wgb_self_attention_noalloc_max_scratch(void) { return wgb::kStaticScratchBytes; }

extern "C" int wgb_self_attention_noalloc(void *attn_val, const void *q, const void *k, const void *v,
                                          wginferDataType_t dtype, size_t seqlen, size_t nhead, size_t nkvhead,
                                          size_t d, size_t dv, size_t total_len, float scale,
                                          wginferStream_t stream) {
    if (seqlen == 0 || nhead == 0) return WGB_OK;
    int rc = wgb::check_args(attn_val, q, k, v, seqlen, nhead, nkvhead, d, dv, total_len, dtype);
    if (rc) return rc;
    const size_t need = wgb_self_attention_workspace_size(seqlen, nhead, nkvhead, d, dv, total_len);
    WGB_REQUIRE(need <= wgb::kStaticScratchBytes, WGB_ERR_OUT_OF_RANGE,
                "wgb_self_attention_noalloc: these sizes need %zu bytes of scratch; the static array holds %zu",
                need, wgb::kStaticScratchBytes);
    void *ws = nullptr;
    if (need) {
        rc = wgb::static_scratch(&ws);
        if (rc) return rc;
    }
    // The scratch holds attn_ref_kernel's one score per key (REFERENCE
    // numerics, caches longer than kRefSmemScores keys). Every score a CTA
    // reads, sc[j] for j < nkeys, is written earlier in the same call, so
    // nothing needs clearing between calls.
    return wgb_self_attention_ex(attn_val, q, k, v, dtype, seqlen, nhead, nkvhead, d, dv, total_len, scale, ws,
                                 need, stream);
}
