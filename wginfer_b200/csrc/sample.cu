// Row-wise top-k / top-p / temperature sampling on the device: the
// reference's host sampler sample_from_logits (src/models/qwen2/model.cpp:
// 60-137), which copies the logits to the host and sorts them, restated for
// one CTA per row with no sort.
//
// Semantics kept from the reference: temperature <= 0, or top_k == 1 with
// top_p >= 1, is the argmax (first index of the maximum); top_k outside
// [1, vocab] means vocab, top_p outside (0, 1] means 1; the candidates are
// the top_k largest logits; the weights are exp(double(f32(l * inv_temp) -
// max_scaled)) with inv_temp = 1.0f / temperature in f32; with top_p < 1 the
// kept set is the shortest prefix, in decreasing logit order, whose weight
// reaches top_p of the candidates' total; the token is drawn from the kept
// set in proportion to the weights. Choices made here: logits that compare
// equal are ordered by index (the reference's partial_sort leaves their
// order unspecified), NaN logits are never candidates unless every logit is
// NaN, and the random number is a counter-based hash of (seed, offset, row)
// (SplitMix64, Steele, Lea and Flood 2014) instead of a host mt19937, so a
// call is reproducible from its seed and offset.
//
// How: order-preserving 32-bit keys of the logits; the k-th largest key by
// a radix select (four passes of 8-bit digits with a shared-memory
// histogram); the top-p threshold by the same select over the weights'
// mass; ties at a threshold are cut by index with a per-warp segment scan.
// Every pass reads the row (L2-resident after the first). Roofline: HBM,
// rows * vocab * size bytes for the first pass; the rest is L2 traffic.
#include "common.cuh"

namespace wgb {
namespace {

constexpr int kST = 1024;         // threads per row
constexpr int kSW = kST / 32;     // warps = index segments

__device__ __forceinline__ uint32_t okey(float v) {
    if (isnan(v)) return 0u;  // below every number
    if (v == 0.f) v = 0.f;    // -0 == +0
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_okey(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ unsigned warp_max_u(unsigned v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// SplitMix64 finaliser of a 64-bit counter.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

struct SampleArgs {
    int64_t *out;
    size_t vocab;
    int top_k;       // in [1, vocab]
    double top_p;    // in (0, 1]
    float inv_temp;  // > 0
    unsigned long long seed, offset;
};

template <typename T>
struct Row {
    const T *x;
    size_t n;
    __device__ __forceinline__ float val(size_t i) const { return Elem<T>::load(x[i]); }
    __device__ __forceinline__ uint32_t key(size_t i) const { return okey(val(i)); }
};

// Radix select over 8-bit digits from the top: among elements with
// in(i, k, w) true, the 32-bit key t at which the running total of w, taken
// from the largest key down, first reaches `need`. *above = the total of w
// over keys strictly above t.
template <typename W, class In>
__device__ uint32_t radix_select(size_t n, In in, W need, W *above, W *hist) {
    __shared__ uint32_t s_digit;
    __shared__ W s_acc;
    uint32_t prefix = 0, mask = 0;
    W acc = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < 256; b += kST) hist[b] = 0;
        __syncthreads();
        for (size_t i = threadIdx.x; i < n; i += kST) {
            uint32_t k;
            W w;
            if (in(i, k, w) && (k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], w);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // lane l owns digits 8l .. 8l + 7; suffix sums from the top
            const int l = threadIdx.x;
            W part = 0;
#pragma unroll
            for (int d = 0; d < 8; d++) part += hist[8 * l + d];
            W suf = part;  // sum over lanes >= l
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const W t = __shfl_down_sync(0xffffffffu, suf, o);
                if (l + o < 32) suf += t;
            }
            const W above_l = suf - part;  // lanes > l
            const bool hit = acc + suf >= need && acc + above_l < need;
            const unsigned hm = __ballot_sync(0xffffffffu, hit);
            // no lane reaches `need` (rounding of the mass): the lowest digit
            const int src = hm ? 31 - __clz(hm) : 0;
            if (l == src) {
                W a = acc + above_l;
                int sel = 8 * l;
                for (int d = 7; d >= 0; d--) {
                    if (a + hist[8 * l + d] >= need || d == 0) {
                        sel = 8 * l + d;
                        break;
                    }
                    a += hist[8 * l + d];
                }
                s_digit = (uint32_t)sel;
                s_acc = a;
            }
        }
        __syncthreads();
        prefix |= s_digit << shift;
        mask |= 255u << shift;
        acc = s_acc;
        __syncthreads();
    }
    *above = acc;
    return prefix;
}

// Index of the `rank`-th (0-based) element, in index order, with key == t
// and in(i); n_seg-element segments per warp.
template <class In>
__device__ size_t nth_tie(size_t n, uint32_t t, In in, unsigned long long rank) {
    __shared__ unsigned long long s_cnt[kSW];
    __shared__ unsigned long long s_idx;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const size_t seg = (n + kSW - 1) / kSW;
    const size_t b = (size_t)w * seg, e = b + seg < n ? b + seg : n;
    unsigned long long c = 0;
    for (size_t i = b + l; i < e; i += 32) {
        uint32_t k;
        double wt;
        if (in(i, k, wt) && k == t) c++;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (l == 0) s_cnt[w] = c;
    if (threadIdx.x == 0) s_idx = n ? n - 1 : 0;
    __syncthreads();
    unsigned long long before = 0;
    for (int q = 0; q < w; q++) before += s_cnt[q];
    if (rank >= before && rank < before + s_cnt[w]) {
        // this warp's segment holds it: scan 32 elements at a time
        unsigned long long r = rank - before;
        for (size_t i0 = b; i0 < e; i0 += 32) {
            const size_t i = i0 + l;
            bool hit = false;
            if (i < e) {
                uint32_t k;
                double wt;
                hit = in(i, k, wt) && k == t;
            }
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            const unsigned cnt = __popc(m);
            if (r < cnt) {
                unsigned mm = m;
                for (unsigned q = 0; q < r; q++) mm &= mm - 1;
                if (l == 0) s_idx = i0 + (__ffs(mm) - 1);
                break;
            }
            r -= cnt;
        }
    }
    __syncthreads();
    return (size_t)s_idx;
}

template <typename T>
__global__ void __launch_bounds__(kST) sample_kernel(const T *logits, SampleArgs a) {
    __shared__ unsigned long long hist_u[256];
    __shared__ double hist_d[256];
    __shared__ uint32_t s_max;
    __shared__ double s_red[kSW];
    const size_t row = blockIdx.x;
    const Row<T> R{logits + row * a.vocab, a.vocab};
    const size_t n = a.vocab;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;

    // maximum key (the first candidate)
    uint32_t mk = 0;
    for (size_t i = threadIdx.x; i < n; i += kST) mk = max(mk, R.key(i));
    mk = warp_max_u(mk);
    if (threadIdx.x == 0) s_max = 0;
    __syncthreads();
    if (l == 0) atomicMax(&s_max, mk);
    __syncthreads();
    const uint32_t kmax = s_max;
    const float max_scaled = __fmul_rn(from_okey(kmax), a.inv_temp);

    // top-k: candidates are keys > tk, and keys == tk up to index ik
    uint32_t tk = 0;
    size_t ik = n;
    if ((size_t)a.top_k < n) {
        unsigned long long above = 0;
        tk = radix_select<unsigned long long>(
            n,
            [&](size_t i, uint32_t &k, unsigned long long &wt) {
                k = R.key(i);
                wt = 1;
                return true;
            },
            (unsigned long long)a.top_k, &above, hist_u);
        const unsigned long long rank = (unsigned long long)a.top_k - above - 1;  // ties kept: rank + 1
        ik = nth_tie(n, tk,
                     [&](size_t i, uint32_t &k, double &wt) {
                         k = R.key(i);
                         wt = 0;
                         return true;
                     },
                     rank);
    }
    // weight of logit v: exp(f32(v * inv_temp) - max_scaled); f32 exp for
    // the selections (accumulated in f64), f64 exp for the draw
    auto wf = [&](float v) -> double { return (double)expf(__fsub_rn(__fmul_rn(v, a.inv_temp), max_scaled)); };
    auto wd = [&](float v) -> double { return exp((double)__fsub_rn(__fmul_rn(v, a.inv_temp), max_scaled)); };
    auto cand = [&](size_t i, uint32_t &k, double &wt) {
        const float v = R.val(i);
        k = okey(v);
        const bool c = (k > tk || (k == tk && i <= ik)) && (k != 0 || kmax == 0);
        wt = c ? wf(v) : 0.0;
        return c;
    };

    // the candidates' total weight
    double tot = 0.0;
    for (size_t i = threadIdx.x; i < n; i += kST) {
        uint32_t k;
        double wt;
        if (cand(i, k, wt)) tot += wt;
    }
    tot = warp_sum_d(tot);
    if (l == 0) s_red[w] = tot;
    __syncthreads();
    tot = 0.0;
    for (int q = 0; q < kSW; q++) tot += s_red[q];
    __syncthreads();

    // top-p: kept = candidates with key > tp, and keys == tp up to index ip
    uint32_t tp = tk;
    size_t ip = ik;
    if (a.top_p < 1.0) {
        double above = 0.0;
        const double need = a.top_p * tot;
        tp = radix_select<double>(n, cand, need, &above, hist_d);
        // ties at tp share one weight; keep the fewest that reach `need`
        const double wt0 = wf(from_okey(tp));
        unsigned long long j = 1;
        if (wt0 > 0.0 && need > above) {
            const double q = ceil((need - above) / wt0);
            j = q < 1.0 ? 1ull : (unsigned long long)q;
        }
        ip = nth_tie(n, tp, cand, j - 1);
    }
    auto kept = [&](size_t i, uint32_t &k, double &wt) {
        const float v = R.val(i);
        k = okey(v);
        const bool kp = (k > tk || (k == tk && i <= ik)) && (k != 0 || kmax == 0) && (k > tp || (k == tp && i <= ip));
        wt = kp ? wd(v) : 0.0;
        return kp;
    };

    // draw: target = u * (kept total); the first index (in index order)
    // whose running sum passes it. Per-warp segments, then one warp scans.
    __shared__ double s_seg[kSW];
    __shared__ unsigned long long s_pick;
    const size_t seg = (n + kSW - 1) / kSW;
    const size_t b = (size_t)w * seg, e = b + seg < n ? b + seg : n;
    double ssum = 0.0;
    for (size_t i = b + l; i < e; i += 32) {
        uint32_t k;
        double wt;
        kept(i, k, wt);
        ssum += wt;
    }
    ssum = warp_sum_d(ssum);
    if (l == 0) s_seg[w] = ssum;
    if (threadIdx.x == 0) s_pick = (unsigned long long)n;
    __syncthreads();
    double kt = 0.0, before = 0.0;
    for (int q = 0; q < kSW; q++) {
        if (q == w) before = kt;
        kt += s_seg[q];
    }
    const uint64_t r = splitmix64(a.seed ^ splitmix64(a.offset * 0x100000001B3ull + row));
    const double u = (double)(r >> 11) * (1.0 / 9007199254740992.0);  // [0, 1)
    const double target = u * kt;
    if (target >= before && target < before + s_seg[w] && s_seg[w] > 0.0) {
        double run = before;
        for (size_t i0 = b; i0 < e; i0 += 32) {
            const size_t i = i0 + l;
            double wt = 0.0;
            if (i < e) {
                uint32_t k;
                kept(i, k, wt);
            }
            // inclusive scan of the 32 weights
            double inc = wt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double t = __shfl_up_sync(0xffffffffu, inc, o);
                if (l >= o) inc += t;
            }
            const unsigned m = __ballot_sync(0xffffffffu, wt > 0.0 && run + inc > target);
            if (m) {
                if (l == 0) s_pick = i0 + (__ffs(m) - 1);
                break;
            }
            run += __shfl_sync(0xffffffffu, inc, 31);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long pick = s_pick;
        if (pick >= n) {
            // rounding left the target past the last kept weight: take the
            // last kept index
            pick = 0;
            for (size_t i = n; i-- > 0;) {
                uint32_t k;
                double wt;
                if (kept(i, k, wt)) {
                    pick = i;
                    break;
                }
            }
        }
        a.out[row] = (int64_t)pick;
    }
}

}  // namespace
}  // namespace wgb

extern "C" int wgb_sample_rows(int64_t *out_idx, const void *logits, wginferDataType_t dtype, size_t rows,
                               size_t vocab, int top_k, float top_p, float temperature, unsigned long long seed,
                               unsigned long long offset, wginferStream_t stream) {
    if (rows == 0) return WGB_OK;
    WGB_REQUIRE(out_idx && logits && vocab > 0, WGB_ERR_INVALID_ARGUMENT, "wgb_sample_rows: null pointer or empty row");
    WGB_REQUIRE(vocab < (1ull << 31) && rows <= (1u << 26), WGB_ERR_INVALID_ARGUMENT, "wgb_sample_rows: size too large");
    // the reference's parameter normalisation (model.cpp:66-81)
    if (!(temperature > 0.0f)) return wgb_argmax_rows(out_idx, nullptr, logits, dtype, rows, vocab, stream);
    if (top_k <= 0 || (size_t)top_k > vocab) top_k = (int)vocab;
    if (!(top_p > 0.0f) || top_p > 1.0f) top_p = 1.0f;
    if (top_k == 1 && top_p >= 1.0f) return wgb_argmax_rows(out_idx, nullptr, logits, dtype, rows, vocab, stream);
    wgb::SampleArgs a;
    a.out = out_idx;
    a.vocab = vocab;
    a.top_k = top_k;
    a.top_p = (double)top_p;
    a.inv_temp = 1.0f / temperature;
    a.seed = seed;
    a.offset = offset;
    cudaStream_t s = (cudaStream_t)stream;
    WGB_DISPATCH_FLOAT(dtype, T,
        wgb::sample_kernel<T><<<(unsigned)rows, wgb::kST, 0, s>>>((const T *)logits, a);
        return wgb::check_launch("wgb_sample_rows"));
    return WGB_OK;
}
