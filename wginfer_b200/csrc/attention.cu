// self_attention: causal GQA attention over a KV cache.
//
// FAST (flash-decode, split-K): a CTA owns one query row, a block of HPC
// heads that share one kv head, and one slice of the visible keys. K/V tiles
// of kKT keys are staged in shared memory once for all HPC heads (GQA
// reuse), scores use an online softmax in f32, and each slice writes
// (max, sum, unnormalised output) to a workspace that a combine kernel folds
// with a log-sum-exp rescale. Slices are chosen so that short queries (decode)
// still fill the SMs. Roofline at decode: HBM, (S*nh*d + 2*L*nkvh*d +
// S*nh*dv) * size bytes.
//
// REFERENCE: one CTA per (query, head) reproduces
// src/ops/self_attention/cpu/self_attention_cpu.cpp:35-89 step for step:
// sequential dot products, -1e9 for masked keys, max, exp, a sequential sum
// over every key, division, and a sequential sum over keys of the rounded
// products p * v.
#include <float.h>

#include "common.cuh"

namespace wgb {
namespace {

constexpr int kKT = 32;       // keys per shared-memory tile
constexpr int kThreads = 256;
constexpr int kMaxAcc = 8;    // output accumulators per thread (HPC*dv <= 2048)

struct AttnShape {
    int S, nh, nkvh, d, dv, L, hpc, nsplit, keys_per_split;
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

// KvCache: batched decode. Query row b is the newest token of sequence
// seq0 + b, whose cache holds lens[b] + 1 positions (its own K/V included);
// it sees all of them.
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

template <typename T, class Src>
__global__ void __launch_bounds__(kThreads) attn_split_kernel(const T *__restrict__ q, Src src, T *__restrict__ out,
                                                              float *__restrict__ ws, AttnShape sh) {
    extern __shared__ float smem[];
    const int dp = sh.d + 1, dvp = sh.dv + 1;
    float *qs = smem;                          // [hpc][d]
    float *ks = qs + sh.hpc * sh.d;            // [kKT][d+1]
    float *vs = ks + kKT * dp;                 // [kKT][dv+1]
    float *ps = vs + kKT * dvp;                // [hpc][kKT]
    float *mrow = ps + sh.hpc * kKT;           // [hpc] running max
    float *lrow = mrow + sh.hpc;               // [hpc] running sum
    float *corr = lrow + sh.hpc;               // [hpc] rescale for this tile

    const int hblocks = sh.nh / sh.hpc;
    const int i = blockIdx.y / hblocks;
    const int hb = blockIdx.y % hblocks;
    const int h0 = hb * sh.hpc;
    const int kvh = h0 * sh.nkvh / sh.nh;
    const int split = blockIdx.x;
    const T *k, *v;
    int nkeys, nvis;
    bool uniform;
    src.row(sh, i, k, v, nkeys, nvis, uniform);
    const int j0 = split * sh.keys_per_split;
    const int j1 = min(j0 + sh.keys_per_split, nvis);
    const int tid = threadIdx.x;

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
    __syncthreads();

    for (int t0 = j0; t0 < j1; t0 += kKT) {
        const int nt = min(kKT, j1 - t0);
        for (int x = tid; x < nt * sh.d; x += kThreads) {
            const int jj = x / sh.d, c = x - jj * sh.d;
            ks[jj * dp + c] = ldf(k, ((size_t)(t0 + jj) * sh.nkvh + kvh) * sh.d + c);
        }
        for (int x = tid; x < nt * sh.dv; x += kThreads) {
            const int jj = x / sh.dv, c = x - jj * sh.dv;
            vs[jj * dvp + c] = ldf(v, ((size_t)(t0 + jj) * sh.nkvh + kvh) * sh.dv + c);
        }
        __syncthreads();
        // scores for hpc x nt
        for (int x = tid; x < sh.hpc * kKT; x += kThreads) {
            const int hh = x / kKT, jj = x - hh * kKT;
            float sc = -FLT_MAX;
            if (jj < nt) {
                if (uniform) {
                    sc = 0.f;
                } else {
                    const float *qq = qs + hh * sh.d;
                    const float *kk = ks + jj * dp;
                    float a = 0.f;
                    for (int c = 0; c < sh.d; c++) a = fmaf(qq[c], kk[c], a);
                    sc = sh.scale * a;
                }
            }
            ps[x] = sc;
        }
        __syncthreads();
        // online softmax update: one warp per head
        const int warp = tid >> 5, lane = tid & 31;
        for (int hh = warp; hh < sh.hpc; hh += kThreads / 32) {
            float sc = lane < nt ? ps[hh * kKT + lane] : -FLT_MAX;
            float mt = warp_max(sc);
            float mold = mrow[hh];
            float mnew = fmaxf(mold, mt);
            float p = lane < nt ? __expf(sc - mnew) : 0.f;
            ps[hh * kKT + lane] = p;
            float sp = warp_sum(p);
            if (lane == 0) {
                float c = __expf(mold - mnew);
                corr[hh] = c;
                lrow[hh] = lrow[hh] * c + sp;
                mrow[hh] = mnew;
            }
        }
        __syncthreads();
#pragma unroll
        for (int a = 0; a < kMaxAcc; a++) {
            const int x = tid + a * kThreads;
            if (x < nacc) {
                const int hh = x / sh.dv, c = x - hh * sh.dv;
                float s = acc[a] * corr[hh];
                const float *pp = ps + hh * kKT;
                for (int jj = 0; jj < nt; jj++) s = fmaf(pp[jj], vs[jj * dvp + c], s);
                acc[a] = s;
            }
        }
        __syncthreads();
    }

    if (sh.nsplit == 1) {
#pragma unroll
        for (int a = 0; a < kMaxAcc; a++) {
            const int x = tid + a * kThreads;
            if (x < nacc) {
                const int hh = x / sh.dv, c = x - hh * sh.dv;
                const float l = lrow[hh];
                stf(out, ((size_t)i * sh.nh + h0 + hh) * sh.dv + c, l > 0.f ? acc[a] / l : 0.f);
            }
        }
        return;
    }
    // workspace: ml[S][nh][nsplit][2], o[S][nh][nsplit][dv]
    float *ml = ws;
    float *o = ws + (size_t)sh.S * sh.nh * sh.nsplit * 2;
    if (tid < sh.hpc) {
        const size_t r = ((size_t)i * sh.nh + h0 + tid) * sh.nsplit + split;
        ml[r * 2] = j0 < j1 ? mrow[tid] : -FLT_MAX;
        ml[r * 2 + 1] = lrow[tid];
    }
#pragma unroll
    for (int a = 0; a < kMaxAcc; a++) {
        const int x = tid + a * kThreads;
        if (x < nacc) {
            const int hh = x / sh.dv, c = x - hh * sh.dv;
            o[(((size_t)i * sh.nh + h0 + hh) * sh.nsplit + split) * sh.dv + c] = acc[a];
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(128) attn_combine_kernel(const float *__restrict__ ws, T *__restrict__ out,
                                                           AttnShape sh) {
    const int row = blockIdx.x;  // i * nh + h
    const float *ml = ws + (size_t)row * sh.nsplit * 2;
    const float *o = ws + (size_t)sh.S * sh.nh * sh.nsplit * 2 + (size_t)row * sh.nsplit * sh.dv;
    float M = -FLT_MAX;
    for (int s = 0; s < sh.nsplit; s++) M = fmaxf(M, ml[2 * s]);
    float L = 0.f;
    for (int s = 0; s < sh.nsplit; s++)
        if (ml[2 * s + 1] > 0.f) L += ml[2 * s + 1] * __expf(ml[2 * s] - M);
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int c = threadIdx.x; c < sh.dv; c += blockDim.x) {
        float a = 0.f;
        for (int s = 0; s < sh.nsplit; s++)
            if (ml[2 * s + 1] > 0.f) a += o[(size_t)s * sh.dv + c] * __expf(ml[2 * s] - M);
        stf(out, (size_t)row * sh.dv + c, a * inv);
    }
}

// ---- REFERENCE order --------------------------------------------------------
template <typename T, class Src>
__global__ void __launch_bounds__(kThreads) attn_ref_kernel(const T *__restrict__ q, Src src, T *__restrict__ out,
                                                            float *__restrict__ gscores, AttnShape sh) {
    extern __shared__ float smem[];
    __shared__ float s_red[kThreads / 32];
    __shared__ float s_max, s_sum;
    const int i = blockIdx.x / sh.nh, h = blockIdx.x % sh.nh;
    const int kvh = h * sh.nkvh / sh.nh;
    float *qs = smem;  // [d]
    float *sc = gscores ? gscores + (size_t)blockIdx.x * sh.L : smem + sh.d;  // [L]
    const int tid = threadIdx.x;
    const T *k, *v;
    int nkeys, nvis;
    bool uniform;
    src.row(sh, i, k, v, nkeys, nvis, uniform);
    for (int c = tid; c < sh.d; c += kThreads) qs[c] = ldf(q, ((size_t)i * sh.nh + h) * sh.d + c);
    __syncthreads();
    // scores: sequential dot, then scale * dot (self_attention_cpu.cpp:37-45)
    for (int j = tid; j < nkeys; j += kThreads) {
        float s = -1e9f;
        if (!uniform && j < nvis) {
            const T *kk = k + ((size_t)j * sh.nkvh + kvh) * sh.d;
            float a = 0.f;
            for (int c = 0; c < sh.d; c++) a = __fadd_rn(a, __fmul_rn(qs[c], ldf(kk, c)));
            s = __fmul_rn(sh.scale, a);
        }
        sc[j] = s;
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
    for (int j = tid; j < nkeys; j += kThreads) sc[j] = exp_cr(__fsub_rn(sc[j], mx));
    __syncthreads();
    if (tid == 0) {  // sequential sum over every key (self_attention_cpu.cpp:70-74)
        float sum = 0.f;
        for (int j = 0; j < nkeys; j++) sum = __fadd_rn(sum, sc[j]);
        s_sum = sum;
    }
    __syncthreads();
    const float sum = s_sum;
    for (int j = tid; j < nkeys; j += kThreads) sc[j] = __fdiv_rn(sc[j], sum);
    __syncthreads();
    // masked keys carry exact zeros and leave the sums unchanged; skip them
    const int jend = nvis;
    for (int c = tid; c < sh.dv; c += kThreads) {
        const T *vv = v + (size_t)kvh * sh.dv + c;
        const size_t vstride = (size_t)sh.nkvh * sh.dv;
        float a = 0.f;
        for (int j = 0; j < jend; j++) a = __fadd_rn(a, __fmul_rn(sc[j], ldf(vv, (size_t)j * vstride)));
        stf(out, ((size_t)i * sh.nh + h) * sh.dv + c, a);
    }
}

constexpr int kRefSmemScores = 11000;  // floats of scores kept in shared memory

int pick_hpc(int G, int dv) {
    for (int h = (G < 8 ? G : 8); h >= 1; h--)
        if (G % h == 0 && h * dv <= kMaxAcc * kThreads && h * kKT <= kThreads) return h;
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
    sh.hpc = pick_hpc((int)(nh / nkvh), (int)dv);
    const long ctas = (long)S * (long)(nh / sh.hpc);
    const long target = 2L * sm_count();
    long ns = ctas >= target ? 1 : (target + ctas - 1) / ctas;
    long max_ns = ((long)L + kKT - 1) / kKT;
    if (ns > max_ns) ns = max_ns;
    if (ns < 1) ns = 1;
    long kps = ((long)L + ns - 1) / ns;
    kps = (kps + kKT - 1) / kKT * kKT;
    ns = ((long)L + kps - 1) / kps;
    sh.nsplit = (int)(ns < 1 ? 1 : ns);
    sh.keys_per_split = (int)kps;
    return sh;
}

size_t ws_bytes(const AttnShape &sh, bool ref) {
    if (ref) return sh.L > kRefSmemScores ? (size_t)sh.S * sh.nh * sh.L * sizeof(float) : 0;
    if (sh.nsplit == 1) return 0;
    return (size_t)sh.S * sh.nh * sh.nsplit * (sh.dv + 2) * sizeof(float);
}

// Raises the dynamic shared-memory limits once per device (a non-stream call,
// kept out of graph capture).
template <typename T, class Src> void set_attrs() {
    cudaFuncSetAttribute(attn_ref_kernel<T, Src>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)((1024 + kRefSmemScores) * sizeof(float)));
    cudaFuncSetAttribute(attn_split_kernel<T, Src>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
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

template <typename T, class Src>
int launch_attn(T *out, const T *q, Src src, const AttnShape &sh, bool ref, void *ws, cudaStream_t s) {
    init_attrs_once();
    if (ref) {
        float *g = sh.L > kRefSmemScores ? (float *)ws : nullptr;
        size_t smem = (size_t)(sh.d + (g ? 0 : sh.L)) * sizeof(float);
        attn_ref_kernel<T, Src><<<sh.S * sh.nh, kThreads, smem, s>>>(q, src, out, g, sh);
        return check_launch("self_attention(reference)");
    }
    size_t smem = (size_t)(sh.hpc * sh.d + kKT * (sh.d + 1) + kKT * (sh.dv + 1) + sh.hpc * kKT + 3 * sh.hpc) * sizeof(float);
    dim3 grid((unsigned)sh.nsplit, (unsigned)(sh.S * (sh.nh / sh.hpc)));
    attn_split_kernel<T, Src><<<grid, kThreads, smem, s>>>(q, src, out, (float *)ws, sh);
    int rc = check_launch("self_attention(split)");
    if (rc || sh.nsplit == 1) return rc;
    attn_combine_kernel<T><<<sh.S * sh.nh, 128, 0, s>>>((const float *)ws, out, sh);
    return check_launch("self_attention(combine)");
}

// Library-owned workspace for the allocation-free-signature entry point.
struct Workspace {
    void *p = nullptr;
    size_t bytes = 0;
};
thread_local Workspace t_ws[64];

int check_args(const void *o, const void *q, const void *k, const void *v, size_t S, size_t nh, size_t nkvh, size_t d,
               size_t dv, size_t L) {
    WGB_REQUIRE(o && q && k && v, WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: null pointer");
    WGB_REQUIRE(nkvh > 0 && nh % nkvh == 0, WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: nhead %% nkvhead != 0");
    WGB_REQUIRE(d > 0 && dv > 0 && d <= 512 && dv <= 512, WGB_ERR_INVALID_ARGUMENT,
                "wgb_self_attention: head dims must be in [1, 512]");
    WGB_REQUIRE(dv <= (size_t)kMaxAcc * kThreads, WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: dv too large");
    WGB_REQUIRE(S < (1u << 20) && L < (1u << 30) && nh < 4096, WGB_ERR_INVALID_ARGUMENT,
                "wgb_self_attention: size too large");
    return WGB_OK;
}

}  // namespace

void attn_prepare() { init_attrs_once(); }

size_t attn_decode_workspace(int B, int nh, int nkvh, int dh, int maxlen, bool ref) {
    AttnShape sh = make_shape((size_t)B, (size_t)nh, (size_t)nkvh, (size_t)dh, (size_t)dh, (size_t)maxlen, 1.f);
    sh.nsplit = (maxlen + sh.keys_per_split - 1) / sh.keys_per_split;
    return ws_bytes(sh, ref);
}

int attn_decode(wginferDataType_t dtype, void *out, const void *q, const void *kcache, const void *vcache,
                size_t seq_stride, const int64_t *lens, int B, int nh, int nkvh, int dh, int maxlen, float scale,
                void *ws, bool ref, cudaStream_t s) {
    // The split count depends only on maxlen, so a captured graph stays valid
    // as the sequences grow; splits past a sequence's length exit at once.
    AttnShape sh = make_shape((size_t)B, (size_t)nh, (size_t)nkvh, (size_t)dh, (size_t)dh, (size_t)maxlen, scale);
    sh.nsplit = (maxlen + sh.keys_per_split - 1) / sh.keys_per_split;
    WGB_DISPATCH_FLOAT(dtype, T,
        return launch_attn((T *)out, (const T *)q,
                           KvCache<T>{(const T *)kcache, (const T *)vcache, seq_stride, lens}, sh, ref, ws, s));
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
    int rc = wgb::check_args(attn_val, q, k, v, seqlen, nhead, nkvhead, d, dv, total_len);
    if (rc) return rc;
    if (total_len == 0) return wgb::set_error(WGB_ERR_INVALID_ARGUMENT, "wgb_self_attention: total_len == 0");
    const bool ref = wgb::current_numerics() == WGB_NUMERICS_REFERENCE;
    wgb::AttnShape sh = wgb::make_shape(seqlen, nhead, nkvhead, d, dv, total_len, scale);
    const size_t need = wgb::ws_bytes(sh, ref);
    WGB_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr), WGB_ERR_INVALID_ARGUMENT,
                "wgb_self_attention_ex: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    WGB_DISPATCH_FLOAT(dtype, T,
        return wgb::launch_attn((T *)attn_val, (const T *)q, wgb::KvDense<T>{(const T *)k, (const T *)v}, sh, ref,
                                workspace, (cudaStream_t)stream));
    return WGB_OK;
}

extern "C" int wgb_self_attention(void *attn_val, const void *q, const void *k, const void *v, wginferDataType_t dtype,
                                  size_t seqlen, size_t nhead, size_t nkvhead, size_t d, size_t dv, size_t total_len,
                                  float scale, wginferStream_t stream) {
    if (seqlen == 0 || nhead == 0) return WGB_OK;
    int rc = wgb::check_args(attn_val, q, k, v, seqlen, nhead, nkvhead, d, dv, total_len);
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
#include <mutex>

namespace wgb {
namespace {

constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB, held by every GPU that loads the library
static __device__ __align__(256) unsigned char g_attn_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void *g_static_ptr[64];  // device address of the array, per device; set once

// The array's name in host code is only a host-side stand-in; the device
// address must be looked up with the device current.
int static_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "wgb_self_attention_noalloc: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(WGB_ERR_INVALID_ARGUMENT, "device id %d", dev);
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (g_static_ptr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess || p == nullptr)
            return set_error(WGB_ERR_CUDA, "wgb_self_attention_noalloc: cudaGetSymbolAddress: %s",
                             cudaGetErrorString(e));
        g_static_ptr[dev] = p;
    }
    *out = g_static_ptr[dev];
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
    int rc = wgb::check_args(attn_val, q, k, v, seqlen, nhead, nkvhead, d, dv, total_len);
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
    // Every scratch word the kernels read is written earlier in the same call
    // (each key slice stores its max, sum and partial output before the
    // combine reads them), so nothing needs clearing between calls.
    return wgb_self_attention_ex(attn_val, q, k, v, dtype, seqlen, nhead, nkvhead, d, dv, total_len, scale, ws,
                                 need, stream);
}
