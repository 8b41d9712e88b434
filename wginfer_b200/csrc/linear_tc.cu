// Tensor-core GEMM for linear with more than 8 input rows (prefill, batched
// decode): out[M, N] = X[M, K] . W[N, K]^T on the 5th-generation tensor cores.
//
// A work unit is 128 weight rows (the MMA's M dimension, one TMEM lane each)
// x TN input rows (the MMA's N dimension, TN in {16, 32, 64, 128, 256}) x a
// range of K; its f32 accumulator [128 x TN] lives in tensor memory. The
// kernel is persistent (one or two CTAs per SM, units strided over the grid) and
// warp-specialised: warp 0 streams 64-wide K slices of W and X into a
// shared-memory ring with TMA (cp.async.bulk.tensor, 128-byte swizzle, no
// multicast); one thread of warp 1 issues tcgen05.mma (kind::f16, bf16 in,
// f32 accumulate, 4 x K16 per slice), frees each stage with tcgen05.commit
// and alternates between two TMEM accumulators; warps 2-5 read a finished
// accumulator with tcgen05.ld (warp w owns TMEM lanes 32 (w % 4) ..., i.e.
// weight rows) and run the same epilogues as the GEMV path
// (decode_common.cuh): bias, residual, SwiGLU of adjacent gate/up rows, or
// RoPE + K/V append of adjacent rotation partners (the partner's value comes
// from the neighbouring lane by shuffle), while the next unit's MMAs fill
// the other accumulator. The epilogue stages each 32-input-row chunk as
// bf16 in shared memory and then writes it (and reads residuals) in 16-byte
// pieces of 8 adjacent outputs. When a tile's weight rows cannot fill the
// GPU (narrow projections), its K range is split over a cluster of CTAs
// whose partial tiles meet in distributed shared memory (plan_split); the
// lm_head of a decode step can fold the greedy argmax into its epilogue
// (EPI_ARGMAX). Roofline: tensor, 2*M*N*K flops (HBM for a few input rows:
// the weights, N*K*2 bytes).
//
// Every mbarrier wait is bounded; on a stall the kernel records an error in
// the device error word, skips the rest, waits (bounded) for copies in
// flight and always releases its tensor memory.
#include <cuda.h>

#include <atomic>

#include "argmax_key.cuh"
#include "common.cuh"
#include "decode_common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace wgb {
namespace {

constexpr int kTcEpiWarps = 4;                     // epilogue warps (one per TMEM lane quarter)
constexpr int kTcThreads = 32 * (2 + kTcEpiWarps);  // + the TMA producer and MMA issuer warps
constexpr int kBK = 64;          // K elements per stage (128 bytes of bf16: one swizzle span)
constexpr int kTcMaxStages = 8;
constexpr int kTileW = 128;      // weight rows per CTA (MMA M)
constexpr int kEpiRows = 32;  // input rows per epilogue chunk
constexpr size_t kEpiTileBytes = (size_t)kEpiRows * kTileW * 2;  // its bf16 staging tile
constexpr int kTcArgmaxRows = 256;  // input rows of a fused lm_head + argmax launch
constexpr int kTcMaxCluster = 16;    // K splits of a tile (a cluster; above 8 where the device allows)
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

// CTAs per SM: two for input tiles up to 64 rows (their MMAs are narrow, and
// a second CTA's MMA and TMA stream interleave with the first's: +5% at 64
// rows of batched decode), else one.
inline int tc_ctas_per_sm(int tn) { return tn <= 64 ? 2 : 1; }
// Stages in the ring: 4 when two CTAs share an SM, else as many as fit in
// about 192 KB, at most kTcMaxStages: 6 for 128 input rows, 4 for 256.
inline int tc_stages(int tn) {
    if (tc_ctas_per_sm(tn) > 1) return 4;
    const int st = kTileW * kBK * 2 + tn * kBK * 2;
    const int n = (192 * 1024) / st;
    return n > kTcMaxStages ? kTcMaxStages : n;
}
inline size_t tc_smem_bytes(int tn) {
    return 1024 + (size_t)tc_stages(tn) * ((size_t)kTileW * kBK * 2 + (size_t)tn * kBK * 2) + kEpiTileBytes;
}
inline size_t tc_smem_max() {
    size_t m = 0;
    for (int tn = 16; tn <= 256; tn *= 2) m = tc_smem_bytes(tn) > m ? tc_smem_bytes(tn) : m;
    return m;
}

// Loads the epilogue issues for a whole chunk before its first store. As
// volatile asm with a memory clobber they stay in program order ahead of the
// stores; as plain loads the compiler sank each one next to its use, behind
// the previous row's stores (which may alias), so the chunk cost one memory
// round trip per row instead of one in all.
__device__ __forceinline__ float ld_bf16_early(const __nv_bfloat16 *p) {
    unsigned short h;
    asm volatile("ld.global.u16 %0, [%1];" : "=h"(h) : "l"(p) : "memory");
    return __uint_as_float((uint32_t)h << 16);
}
__device__ __forceinline__ uint4 ld_global_v4_early(const void *p) {
    uint4 r;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ int64_t ld_s64_early(const int64_t *p) {
    long long v;
    asm volatile("ld.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return (int64_t)v;
}

// The epilogue of a chunk of up to 32 input rows runs in two phases through
// a shared-memory tile S[32][128] of bf16 (input row j, weight row r):
//   stage: each epilogue thread owns one weight row (its TMEM lane) and
//          writes round(sum + bias) for the chunk's input rows (one column
//          of S per thread: conflict-free);
//   emit:  the 128 threads then take 16-byte pieces of S rows (8 adjacent
//          weight rows of one input row), so residual loads and output
//          stores are coalesced 16-byte accesses, all loads of a thread
//          requested before its first store.
// (A thread that walked its 32 input rows itself issued scattered 2-byte
// accesses one row at a time; that cost one memory round trip per row.)
// The RoPE piece hoists everything that depends only on the weight rows
// (head, rotation index, q/k/v) out of the loop over input rows.

__device__ __forceinline__ void tc_epi_stage(__nv_bfloat16 *S, int row, const float (&v)[32], float b) {
#pragma unroll
    for (int j = 0; j < kEpiRows; j++) S[j * kTileW + row] = __float2bfloat16_rn(v[j] + b);
}

template <int EPI>
__device__ __forceinline__ void tc_epi_emit(const DecodeGemvParams &p, const __nv_bfloat16 *S, int n0, int mc,
                                            int cols, int et, unsigned long long *s_key = nullptr) {
    using T = __nv_bfloat16;
    constexpr int kPer = kEpiRows * kTileW / 8 / (kTcEpiWarps * 32);  // 16-byte pieces per thread (4)
    const int nc = (et & 15) * 8;                                        // first weight row of the piece
    const int jb = et >> 4;                                              // input rows jb, jb + 8, ...
    Vec16<T> sv[kPer];
#pragma unroll
    for (int k = 0; k < kPer; k++) sv[k].u = *reinterpret_cast<const uint4 *>(S + (jb + 8 * k) * kTileW + nc);
    if constexpr (EPI == EPI_ARGMAX) {
        // lm_head + greedy argmax: the logits are stored as they are, and each
        // input row's best (value, first index) key over this thread's 8
        // weight rows is folded over the 16 threads of the row, then into the
        // CTA's key for the row (argmax_key.cuh)
        T *out = reinterpret_cast<T *>(p.out);
        const bool vec = n0 + nc + 8 <= p.N && (p.ldo & 7) == 0 && ((uintptr_t)out & 15) == 0;
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = jb + 8 * k, m = mc + j;
            const bool live = j < cols && m < p.M;
            unsigned long long key = 0ull;
            if (live) {
                const size_t off = (size_t)m * p.ldo + n0 + nc;
                if (vec) *reinterpret_cast<uint4 *>(out + off) = sv[k].u;
                // the vector's largest value (NaN never wins: fmaxf skips
                // it) and its first index (-0 and +0 compare equal), then one
                // key for the vector instead of one per logit (the epilogue
                // of a 64 x 128 unit: 6.7 -> 5.6 us)
                float mx = -INFINITY;
                int first = -1;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    if (n0 + nc + e < p.N) {
                        if (!vec) out[off + e] = sv[k].e[e];
                        mx = fmaxf(mx, Elem<T>::load(sv[k].e[e]));
                    }
                }
#pragma unroll
                for (int e = 7; e >= 0; e--)
                    if (n0 + nc + e < p.N && Elem<T>::load(sv[k].e[e]) == mx) first = e;
                if (first >= 0) key = make_key(mx, (uint32_t)(n0 + nc + first));
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            if (live && (et & 15) == 0 && key) atomicMax(&s_key[m], key);
        }
    } else if constexpr (EPI == EPI_STORE) {
        T *out = reinterpret_cast<T *>(p.out);
        const T *res = reinterpret_cast<const T *>(p.res);
        const bool vec = n0 + nc + 8 <= p.N && (p.ldo & 7) == 0 && ((uintptr_t)out & 15) == 0 &&
                         ((uintptr_t)res & 15) == 0;
        Vec16<T> rv[kPer];
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = jb + 8 * k, m = mc + j;
            rv[k].u = make_uint4(0, 0, 0, 0);
            if (res && j < cols && m < p.M) {
                const size_t o = (size_t)m * p.ldo + n0 + nc;
                if (vec) {
                    rv[k].u = ld_global_v4_early(res + o);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        if (n0 + nc + e < p.N) rv[k].e[e] = __float2bfloat16_rn(ld_bf16_early(res + o + e));
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = jb + 8 * k, m = mc + j;
            if (j >= cols || m >= p.M) continue;
            Vec16<T> o;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float x = Elem<T>::load(sv[k].e[e]);
                o.e[e] = res ? __float2bfloat16_rn(__fadd_rn(Elem<T>::load(rv[k].e[e]), x)) : sv[k].e[e];
            }
            const size_t off = (size_t)m * p.ldo + n0 + nc;
            if (vec) {
                *reinterpret_cast<uint4 *>(out + off) = o.u;
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++)
                    if (n0 + nc + e < p.N) out[off + e] = o.e[e];
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        // rows (2g, 2g + 1) are gate and up of output g
        T *out = reinterpret_cast<T *>(p.out);
        const int g0 = (n0 + nc) >> 1;
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = jb + 8 * k, m = mc + j;
            if (j >= cols || m >= p.M) continue;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                if (n0 + nc + 2 * q >= p.N) continue;  // the pair's gate row lies past N
                const float gg = Elem<T>::load(sv[k].e[2 * q]);
                const float uu = Elem<T>::load(sv[k].e[2 * q + 1]);
                stf(out, (size_t)m * p.ldo + g0 + q, __fdiv_rn(__fmul_rn(uu, gg), __fadd_rn(1.0f, expf(-gg))));
            }
        }
    } else {
        // RoPE + K/V append. A piece is four row pairs g0 .. g0 + 3 of one
        // head (q or k: rotation partners (jj, jj + dh/2), jj = g0 % (dh/2) ..
        // + 3) or eight consecutive v values; per input row: its position,
        // four {cos, sin} (32 bytes) and two 8-byte stores (q, k) or one
        // 16-byte store (v).
        const int half = p.dh >> 1;
        const int P = (p.nh + p.nkvh) * half;
        const int g0 = (n0 + nc) >> 1;
        const bool qk = g0 < P;
        const int h = g0 / half, jj0 = g0 - h * half, e0 = 2 * (g0 - P);
        const bool vec = n0 + nc + 8 <= p.N && (half & 3) == 0 && (p.dh & 7) == 0 && (P & 3) == 0 &&
                         ((uintptr_t)p.q_out & 15) == 0 && ((uintptr_t)p.kc & 15) == 0 &&
                         ((uintptr_t)p.vc & 15) == 0 && ((uintptr_t)p.table & 15) == 0 && (p.seq_stride & 7) == 0;
        int64_t pos[kPer];
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = jb + 8 * k, m = mc + j;
            pos[k] = j < cols && m < p.M ? ld_s64_early(p.pos + m) : -1;
        }
        if (!vec) {  // ragged or unaligned: one pair at a time
#pragma unroll
            for (int k = 0; k < kPer; k++) {
                const int j = jb + 8 * k, m = mc + j;
                if (j >= cols || m >= p.M) continue;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int r0 = n0 + nc + 2 * q, g = g0 + q;
                    if (r0 >= p.N) continue;
                    float2 cs = make_float2(0.f, 0.f);
                    if (g < P && pos[k] >= 0 && pos[k] < p.maxseq) cs = p.table[(size_t)pos[k] * half + (g % half)];
                    rope_kv_store<T>(p, g, r0 + 1 < p.N, m, Elem<T>::load(sv[k].e[2 * q]),
                                     Elem<T>::load(sv[k].e[2 * q + 1]), pos[k], cs);
                }
            }
            return;
        }
        float4 cs[kPer][2];
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            cs[k][0] = cs[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (qk && pos[k] >= 0 && pos[k] < p.maxseq) {
                const float2 *c = p.table + (size_t)pos[k] * half + jj0;
                const uint4 a = ld_global_v4_early(c), b = ld_global_v4_early(c + 2);
                cs[k][0] = make_float4(__uint_as_float(a.x), __uint_as_float(a.y), __uint_as_float(a.z),
                                       __uint_as_float(a.w));
                cs[k][1] = make_float4(__uint_as_float(b.x), __uint_as_float(b.y), __uint_as_float(b.z),
                                       __uint_as_float(b.w));
            }
        }
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = jb + 8 * k, m = mc + j;
            if (j >= cols || m >= p.M) continue;
            if (pos[k] < 0 || pos[k] >= p.maxseq) {
                record_device_error(p.err, 3, pos[k]);
                continue;
            }
            const int seq = p.prefill_seq >= 0 ? p.prefill_seq : m;
            const size_t cache = (size_t)seq * p.seq_stride + (size_t)pos[k] * p.nkvh * p.dh;
            if (qk) {
                T *dst = h < p.nh ? reinterpret_cast<T *>(p.q_out) + ((size_t)m * p.nh + h) * p.dh
                                  : reinterpret_cast<T *>(p.kc) + cache + (size_t)(h - p.nh) * p.dh;
                const float c4[4] = {cs[k][0].x, cs[k][0].z, cs[k][1].x, cs[k][1].z};
                const float s4[4] = {cs[k][0].y, cs[k][0].w, cs[k][1].y, cs[k][1].w};
                union { uint2 u; T e[4]; } lo, hi;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float a = Elem<T>::load(sv[k].e[2 * q]), b = Elem<T>::load(sv[k].e[2 * q + 1]);
                    lo.e[q] = Elem<T>::store(__fsub_rn(__fmul_rn(a, c4[q]), __fmul_rn(b, s4[q])));
                    hi.e[q] = Elem<T>::store(__fadd_rn(__fmul_rn(a, s4[q]), __fmul_rn(b, c4[q])));
                }
                *reinterpret_cast<uint2 *>(dst + jj0) = lo.u;
                *reinterpret_cast<uint2 *>(dst + jj0 + half) = hi.u;
            } else {
                *reinterpret_cast<uint4 *>(reinterpret_cast<T *>(p.vc) + cache + e0) = sv[k].u;
            }
        }
    }
}

// Work units of one launch: output tile t = (weight tile bx, input tile by)
// and K split z; unit u = (t * ksplit + z), t = bx * tiles_m + by, so the
// input tiles that share a weight tile (and the K splits of a tile) run on
// neighbouring CTAs at the same time.
struct TcSched {
    int tiles_m, ksplit, kper, ktiles_total, nunits;
    __device__ __forceinline__ void unit(int u, int tn, int &t, int &n0, int &m0, int &kb, int &nk) const {
        const int z = u % ksplit;
        t = u / ksplit;
        n0 = (t / tiles_m) * kTileW;
        m0 = (t % tiles_m) * tn;
        kb = z * kper;
        nk = min(kper, ktiles_total - kb);
    }
};

// Cluster barrier over every thread of every CTA of the cluster (release /
// acquire: shared-memory writes before it are visible to the cluster after).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kTcEpiWarps * 32) : "memory"); }
__device__ __forceinline__ void mb_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s_u32(b)) : "memory");
}

// Persistent and warp-specialised: warp 0 streams the K slices of this CTA's
// units through the shared-memory ring (TMA), warp 1 issues the MMAs of
// unit i into TMEM accumulator i % 2, warps 2-5 run the epilogue of unit i
// from that accumulator while the MMAs of unit i + 1 fill the other one.
// Warp w of the epilogue reads TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31.
template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, DecodeGemvParams p,
                   int tn, int nst, TcSched sc) {
    using T = __nv_bfloat16;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[kTcMaxStages], empty[kTcMaxStages], acc_full[2], acc_empty[2], done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_bad, s_issued, s_last, s_stop[2];
    __shared__ unsigned long long s_key[EPI == EPI_ARGMAX ? kTcArgmaxRows : 1];  // this CTA's best key per input row
    unsigned char *smem = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int a_bytes = kTileW * kBK * 2, b_bytes = tn * kBK * 2, st_bytes = a_bytes + b_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ncols = tn <= 32 ? 32 : (uint32_t)tn;  // columns of one accumulator (a power of two >= 32)

    if (threadIdx.x == 0) {
        s_bad = 0;
        s_issued = 0;
        for (int i = 0; i < nst; i++) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mb_init(&acc_full[i], 1);
            mb_init(&acc_empty[i], kTcEpiWarps);
        }
        mb_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(&s_tmem)),
                     "r"(2 * ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // producer: TMA slices of W (128 rows) and X (tn rows) into the
            // ring. The weights of the first stages do not depend on the
            // previous kernel: they are requested before the wait for it;
            // X (written by it) right after.
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmW) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmX) : "memory");
            int pre = 0, m0f = 0, kbf = 0;
            if ((int)blockIdx.x < sc.nunits) {
                int t, n0, nk;
                sc.unit(blockIdx.x, tn, t, n0, m0f, kbf, nk);
                pre = min(nk, nst);
                for (int kt = 0; kt < pre; kt++) {
                    mb_expect_tx(&full[kt], (unsigned)st_bytes);
                    tma_load_2d(smem + (size_t)kt * st_bytes, &tmW, (kbf + kt) * kBK, n0, &full[kt]);
                }
            }
            pdl_wait();
            for (int kt = 0; kt < pre; kt++)
                tma_load_2d(smem + (size_t)kt * st_bytes + a_bytes, &tmX, (kbf + kt) * kBK, m0f, &full[kt]);
            s_issued = pre;
            int it = 0;
            for (int u = blockIdx.x; u < sc.nunits; u += gridDim.x) {
                int t, n0, m0, kb, nk;
                sc.unit(u, tn, t, n0, m0, kb, nk);
                for (int kt = 0; kt < nk; kt++, it++) {
                    if (it < pre) continue;  // issued above
                    const int st = it % nst;
                    if (it >= nst && !mb_wait(&empty[st], (unsigned)(((it / nst) - 1) & 1))) {
                        atomicExch(&s_bad, 1);
                        break;
                    }
                    unsigned char *a = smem + (size_t)st * st_bytes;
                    mb_expect_tx(&full[st], (unsigned)st_bytes);
                    tma_load_2d(a, &tmW, (kb + kt) * kBK, n0, &full[st]);
                    tma_load_2d(a + a_bytes, &tmX, (kb + kt) * kBK, m0, &full[st]);
                    s_issued = it + 1;
                }
                if (*(volatile int *)&s_bad) break;
            }
        }
    } else if (warp == 1) {
        // (reads only shared memory that the producer fills after its wait)
        if (lane == 0) {
            // MMA issuer
            const uint32_t idesc = idesc_bf16(tn);
            int it = 0, i = 0;
            for (int u = blockIdx.x; u < sc.nunits; u += gridDim.x, i++) {
                int t, n0, m0, kb, nk;
                sc.unit(u, tn, t, n0, m0, kb, nk);
                const int buf = i & 1, use = i >> 1;
                if (use >= 1 && !mb_wait(&acc_empty[buf], (unsigned)((use - 1) & 1))) {
                    atomicExch(&s_bad, 1);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + (uint32_t)buf * ncols;
                bool ok = true;
                for (int kt = 0; kt < nk; kt++, it++) {
                    const int st = it % nst;
                    if (!mb_wait(&full[st], (unsigned)((it / nst) & 1))) {
                        atomicExch(&s_bad, 1);
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const unsigned char *a = smem + (size_t)st * st_bytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        mma_bf16(d, sw128_desc(a + k * 32), sw128_desc(a + a_bytes + k * 32), idesc, (kt | k) != 0);
                    mma_commit(&empty[st]);  // the stage is free once these MMAs have read it
                }
                if (!ok) break;
                mma_commit(&acc_full[buf]);  // the accumulator is complete once they have run
            }
            mma_commit(&done);
        }
    } else {
        // epilogue warps
        pdl_wait();  // residuals (and the output) come from earlier kernels
        const int q = warp & 3;  // TMEM lane quarter
        const int row = q * 32 + lane;
        const int et = threadIdx.x - 64;  // 0 .. 127 among the epilogue threads
        __nv_bfloat16 *S = reinterpret_cast<__nv_bfloat16 *>(smem + (size_t)nst * st_bytes);
        const bool leader = warp == 2 && lane == 0;
        if constexpr (EPI == EPI_ARGMAX)
            for (int m = et; m < kTcArgmaxRows; m += kTcEpiWarps * 32) s_key[m] = 0ull;  // ordered by epi_bar below
        int i = 0;
        for (int u = blockIdx.x; u < sc.nunits; u += gridDim.x, i++) {
            int t, n0, m0, kb, nk;
            sc.unit(u, tn, t, n0, m0, kb, nk);
            const int buf = i & 1, use = i >> 1;
            // one thread waits for the accumulator; the decision to go on is
            // shared through s_stop so the four warps never part at a barrier
            if (leader) s_stop[i & 1] = !mb_wait(&acc_full[buf], (unsigned)(use & 1)) || *(volatile int *)&s_bad;
            epi_bar();
            if (s_stop[i & 1]) {
                if (leader) atomicExch(&s_bad, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)buf * ncols;
            const int n = n0 + row;
            // this weight row's bias, loaded once per unit
            const float brow = p.bias && n < p.N ? ldf(reinterpret_cast<const T *>(p.bias), n) : 0.f;
            if (sc.ksplit > 1) {
                // split-K: this CTA's partial tile ([tn][128] f32, weight
                // rows contiguous) goes to its own shared memory, over the
                // ring (idle: the CTA's only unit has been read by its MMAs);
                // the cluster reduces the tile after the role branches
                float *P = reinterpret_cast<float *>(smem);
                for (int c0 = 0; c0 < tn; c0 += 32) {
                    uint32_t r[32];
                    tmem_ld32(acc + (uint32_t)c0, r);
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (c0 + j < tn) P[(size_t)(c0 + j) * kTileW + row] = __uint_as_float(r[j]);
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mb_arrive(&acc_empty[buf]);
            } else {
                for (int c0 = 0; c0 < tn; c0 += 32) {
                    uint32_t r[32];
                    tmem_ld32(acc + (uint32_t)c0, r);
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                    if (c0 + 32 >= tn) {  // last chunk read: the MMAs may refill this accumulator
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mb_arrive(&acc_empty[buf]);
                    }
                    tc_epi_stage(S, row, v, brow);
                    epi_bar();
                    tc_epi_emit<EPI>(p, S, n0, m0 + c0, min(32, tn - c0), et, s_key);
                    epi_bar();  // S is rewritten by the next chunk
                }
            }
        }
        if constexpr (EPI == EPI_ARGMAX) {
            // every CTA merges its keys (one global atomic per input row) and
            // arrives, also after a stall; the last to arrive turns the keys
            // into tokens, advances the lengths (model.cpp:398-407) and
            // clears the keys and the counter for the next launch
            epi_bar();
            for (int m = et; m < p.M; m += kTcEpiWarps * 32)
                if (s_key[m]) atomicMax(&p.amax_keys[m], s_key[m]);
            __threadfence();
            epi_bar();
            if (leader) s_last = atomicAdd(p.amax_count, 1u) == gridDim.x - 1;
            epi_bar();
            if (s_last) {
                __threadfence();
                for (int m = et; m < p.M; m += kTcEpiWarps * 32) {
                    const unsigned long long key = atomicExch(&p.amax_keys[m], 0ull);
                    const unsigned short u0 = __ldcg(reinterpret_cast<const unsigned short *>(p.out) + (size_t)m * p.ldo);
                    p.tokens[m] = key_index(key, __uint_as_float((uint32_t)u0 << 16));
                    if (p.lens && p.lens[m] < p.maxlen) p.lens[m] += 1;
                }
                epi_bar();
                if (leader) atomicExch(p.amax_count, 0u);
            }
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
        // every MMA this CTA issued has completed (tracked by `done`)
        if (!mb_wait(&done, 0)) s_bad = 1;
        if (s_bad) {
            record_device_error(p.err, 6, blockIdx.x);
            // TMA copies may still be landing in the ring: wait (bounded) for
            // the last one issued into each stage before the CTA exits
            for (int it = s_issued - 1; it >= 0 && it >= s_issued - nst; it--)
                mb_wait(&full[it % nst], (unsigned)((it / nst) & 1));
        }
    }
    __syncthreads();
    if (sc.ksplit > 1) {
        // split-K over the cluster (the tile's K splits are its consecutive
        // CTAs, one unit each): every partial tile is in its CTA's shared
        // memory; CTA z adds the ksplit partials of input rows
        // [z * per, (z + 1) * per) in split order (a fixed order, so results
        // do not vary from run to run) through distributed shared memory and
        // runs the epilogue for them; a second cluster barrier keeps every
        // CTA's partial tile alive until all have read it
        cluster_sync_all();
        if (warp >= 2) {
            // thread et adds weight rows r4 .. r4 + 3 (one 16-byte load per
            // split) of input rows jo, jo + 4, ...: four rows of the tile per
            // pass of the 128 threads
            const int et = threadIdx.x - 64, r4 = (et & 31) * 4, jo = et >> 5;
            const int z = (int)cluster_rank();
            const int per = (tn + sc.ksplit - 1) / sc.ksplit;
            const int j0 = min(tn, z * per), j1 = min(tn, j0 + per);
            int t, n0, m0, kb, nk;
            sc.unit(blockIdx.x, tn, t, n0, m0, kb, nk);
            float brow[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int n = n0 + r4 + i;
                brow[i] = p.bias && n < p.N ? ldf(reinterpret_cast<const T *>(p.bias), n) : 0.f;
            }
            __nv_bfloat16 *S = reinterpret_cast<__nv_bfloat16 *>(smem + (size_t)nst * st_bytes);
            uint32_t pq[kTcMaxCluster];  // each split's partial tile, as a cluster shared address
#pragma unroll
            for (int q = 0; q < kTcMaxCluster; q++) pq[q] = q < sc.ksplit ? cluster_map(s_u32(smem), q) : 0u;
            for (int jc = j0; jc < j1; jc += kEpiRows) {
                const int nr = min(kEpiRows, j1 - jc);
                for (int j = jo; j < nr; j += 4) {
                    const uint32_t off = (uint32_t)(((jc + j) * kTileW + r4) * 4);
                    float4 x[kTcMaxCluster];
#pragma unroll
                    for (int q = 0; q < kTcMaxCluster; q++)
                        x[q] = q < sc.ksplit ? ld_cluster_f32x4(pq[q] + off) : make_float4(0.f, 0.f, 0.f, 0.f);
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int q = 0; q < kTcMaxCluster; q++) {  // in split order: the same bits on every run
                        acc.x += x[q].x;
                        acc.y += x[q].y;
                        acc.z += x[q].z;
                        acc.w += x[q].w;
                    }
                    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x + brow[0], acc.y + brow[1]);
                    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z + brow[2], acc.w + brow[3]);
                    uint2 pk;
                    pk.x = *reinterpret_cast<uint32_t *>(&lo);
                    pk.y = *reinterpret_cast<uint32_t *>(&hi);
                    *reinterpret_cast<uint2 *>(S + j * kTileW + r4) = pk;
                }
                epi_bar();
                tc_epi_emit<EPI>(p, S, n0, m0 + jc, nr, et, s_key);
                epi_bar();  // S is rewritten by the next chunk
            }
        }
        cluster_sync_all();
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * ncols) : "memory");
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

}  // namespace

bool tma_map_rows(CUtensorMap *tm, const void *base, int es, int rows, int cols, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (es != 2 && es != 4)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * (cuuint64_t)es};
    cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(tm, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tma_map_row_stages(CUtensorMap *tm, const void *base, int es, int rows, int cols, int box_rows, int stages) {
    EncodeTiledFn fn = encode_fn();
    const int blk = es == 2 || es == 4 ? 128 / es : 0;
    if (!fn || !blk || cols % blk) return false;
    cuuint64_t dims[3] = {(cuuint64_t)blk, (cuuint64_t)rows, (cuuint64_t)(cols / blk)};
    cuuint64_t strides[2] = {(cuuint64_t)cols * (cuuint64_t)es, 128};
    cuuint32_t box[3] = {(cuuint32_t)blk, (cuuint32_t)box_rows, (cuuint32_t)stages};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(tm, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

// Input rows per tile: the smallest power of two >= M up to 256 (the MMA's
// largest N; fewer re-reads of the weight tile), then halved (down to 16)
// only while the grid would leave more than half the CTA slots idle (two per
// SM for tiles up to 64 rows): each halving
// re-reads the weights once more (from L2) and makes every MMA narrower.
// (Choosing instead, above 128 rows, the tile with the fewest operand bytes
// per SM, 64-row tiles for q/k/v, o and down at 512 rows, measured slower:
// 4.74 against 4.63 ms for the 512-token prefill; a unit with a long K range
// is bound by the bytes its ring keeps in flight, not by L2.)
int pick_tn(int M, int N) {
    int tn = 16;
    while (tn < M && tn < 256) tn *= 2;
    const long long wtiles = (N + kTileW - 1) / kTileW;
    while (tn > 16 && 2 * wtiles * ((M + tn - 1) / tn) <= (long long)sm_count() * tc_ctas_per_sm(tn / 2)) tn /= 2;
    return tn;
}

// Split-K plan: when the weight tiles of the widest input tile cannot fill
// half the SMs, keep that tile (the weights are read once, and wide MMAs)
// and split K across a cluster of CTAs instead, as many splits as fit in one
// wave, at most the largest cluster the device schedules for that launch
// (max_cluster); the partial tiles meet in distributed shared memory.
// Otherwise ksplit = 1 and the input tile comes from pick_tn.
// Up to 128 input rows (q/k/v, o and down at batch 64, prefill chunks of up
// to 128 tokens) every such projection splits. Above, a 256-row input tile's
// partial (128 KB of f32 per CTA) makes the cluster reduction cost more than
// the unsplit plan's narrower input tiles unless K is long and the split is
// at least 4 ways; of the Qwen2-1.5B shapes that keeps only down (K = 8960)
// split, at 256 and 512 rows. Measured on the 28-layer prefill (ms; every
// projection split / none split / down split only): 128 tokens 3.09-3.15 /
// 3.53 / -, 256 tokens 4.08 / 3.93 / 3.24, 512 tokens 5.39-5.41 / 4.63-4.66 /
// 4.43; at 1024 tokens down splits 3 ways: 7.06 split against 6.33 unsplit.
// (Splitting gate/up at batch 64 in two, instead of two 32-row input tiles,
// measured 27.6 against 22.5 us serialised.)
void plan_split(const DecodeGemvParams &p, bool allow_split, int max_cluster, int &tn, int &ksplit, int &kper) {
    const int ktiles = (p.K + kBK - 1) / kBK;
    ksplit = 1;
    kper = ktiles;
    int wide = 16;
    while (wide < p.M && wide < 256) wide *= 2;
    const long long tiles = (long long)((p.N + kTileW - 1) / kTileW) * ((p.M + wide - 1) / wide);
    const long long sms = sm_count(), slots = sms * tc_ctas_per_sm(wide);  // CTAs of one wave
    const bool long_k = ktiles >= 128 && 4 * tiles <= slots;
    if (allow_split && (wide <= 128 || long_k) && 2 * tiles <= sms && ktiles >= 2) {
        int ks = (int)(slots / tiles);
        if (ks > ktiles) ks = ktiles;
        if (ks > max_cluster) ks = max_cluster;
        const int per = (ktiles + ks - 1) / ks;
        ks = (ktiles + per - 1) / per;  // every split gets at least one slice
        if (ks > 1) {
            tn = wide;
            ksplit = ks;
            kper = per;
            return;
        }
    }
    tn = pick_tn(p.M, p.N);
}

// Largest cluster of split-K CTAs the device schedules for this kernel at
// the widest split-K tile (64 input rows, two CTAs per SM), at most
// kTcMaxCluster; clusters above 8 need the non-portable size attribute. The
// function attributes are set here (a non-stream call, kept out of graph
// capture by the first launch).
template <int EPI> int tc_max_cluster() {
    static std::atomic<int> cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64) {
        const int c = cache[dev].load(std::memory_order_acquire);
        if (c) return c;
    }
    cudaFuncSetAttribute(tc_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_max());
    int best = 8;
    if (cudaFuncSetAttribute(tc_gemm_kernel<EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kTcMaxCluster);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = tc_smem_bytes(64);
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = kTcMaxCluster;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxPotentialClusterSize(&n, tc_gemm_kernel<EPI>, &cfg) == cudaSuccess && n > best) best = n;
    }
    cudaGetLastError();
    if (best > kTcMaxCluster) best = kTcMaxCluster;
    if (dev >= 0 && dev < 64) cache[dev].store(best, std::memory_order_release);
    return best;
}

template <int EPI>
int launch_tc(const DecodeGemvParams &p, cudaStream_t s) {
    int tn, ksplit, kper;
    plan_split(p, EPI != EPI_ARGMAX, tc_max_cluster<EPI>(), tn, ksplit, kper);
    TcSched sc;
    sc.tiles_m = (p.M + tn - 1) / tn;
    sc.ksplit = ksplit;
    sc.kper = kper;
    sc.ktiles_total = (p.K + kBK - 1) / kBK;
    const long long units = (long long)((p.N + kTileW - 1) / kTileW) * sc.tiles_m * ksplit;
    if (units > (1ll << 30)) return set_error(WGB_ERR_INVALID_ARGUMENT, "linear(tc): too many tiles");
    sc.nunits = (int)units;
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
    // persistent: one or two CTAs per SM (the ring takes most of the shared
    // memory), each taking units blockIdx.x, blockIdx.x + gridDim.x, ...;
    // split-K: one unit per CTA (the plan keeps them within one wave), the
    // K splits of a tile as one cluster
    const int cap = sm_count() * tc_ctas_per_sm(tn);
    if (ksplit > 1 && sc.nunits > cap) return set_error(WGB_ERR_UNSUPPORTED, "linear(tc): split-K plan exceeds one wave");
    cfg.gridDim = dim3((unsigned)(sc.nunits < cap ? sc.nunits : cap));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = tc_smem_bytes(tn);
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl_enabled()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (ksplit > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = (unsigned)ksplit;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<EPI>, tmW, tmX, p, tn, tc_stages(tn), sc);
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "linear(tc): %s", cudaGetErrorString(e));
    return WGB_OK;
}

}  // namespace

bool tc_gemm_ok(const DecodeGemvParams &p) {
    // TMA: 16-byte aligned bases and row strides
    return p.M > 8 && p.K > 0 && p.K % 8 == 0 && aligned16(p.w) && aligned16(p.x) && p.N >= 1 && encode_fn() &&
           p.M <= 128 * 65535 && p.N < (1 << 30);
}

int tc_gemm(const DecodeGemvParams &p0, int epi, cudaStream_t s) {
    DecodeGemvParams p = p0;
    if (!p.err) p.err = dev_error_ptr();  // stalls are reported through the device error word
    if (epi == DG_EPI_SWIGLU) return launch_tc<EPI_SWIGLU>(p, s);
    if (epi == DG_EPI_ROPEKV) return launch_tc<EPI_ROPEKV>(p, s);
    if (epi == DG_EPI_ARGMAX) {
        WGB_REQUIRE(p.M <= kTcArgmaxRows && !p.bias && !p.res && p.amax_keys && p.amax_count && p.tokens && p.out,
                    WGB_ERR_INVALID_ARGUMENT, "linear(tc): argmax epilogue needs <= %d rows, its key buffers, no bias",
                    kTcArgmaxRows);
        return launch_tc<EPI_ARGMAX>(p, s);
    }
    return launch_tc<EPI_STORE>(p, s);
}

void tc_gemm_prepare() {
    const int lim = (int)tc_smem_max();
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_ROPEKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(tc_gemm_kernel<EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    tc_max_cluster<EPI_STORE>();  // the cluster limits are settled outside any graph capture
    tc_max_cluster<EPI_SWIGLU>();
    tc_max_cluster<EPI_ROPEKV>();
    tc_max_cluster<EPI_ARGMAX>();
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
