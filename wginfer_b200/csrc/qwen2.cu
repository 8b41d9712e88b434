// Qwen2 decoder on the B200 backend: the caller of the decode-path ops.
//
// Follows src/models/qwen2/model.cpp (forward_layer :243-328, forward
// :331-368, infer :371-415) with the same op sequence and rounding points,
// re-planned for the device:
//  - one device arena holds weights, per-sequence KV caches and activations;
//  - q/k/v weights (and biases) are stored as one [(nh + 2 nkvh) dh, hs]
//    matrix and gate/up as one [2 di, hs] matrix, so each is one GEMV; each
//    output row is still its own dot product, so results are unchanged;
//  - RoPE, the K/V cache append (the reference's two synchronous D2D copies)
//    and the q copy are one kernel reading a cos/sin table built on the host
//    with the reference's exact formula (rope_cpu.cpp:13-30);
//  - the residual adds are fused into the o_proj and down_proj epilogues
//    (round(x + round(W a)), the reference's linear-then-add);
//  - logits are formed for the last prompt row only (the reference computes
//    every row and reads the last, model.cpp:363-396);
//  - greedy argmax stays on the device; a decode step for a batch of
//    sequences reads and writes a device token buffer and is captured once
//    into a CUDA graph, so a step costs one graph launch and no host sync.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <random>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace wgb {
namespace {

size_t dsize(int dt) { return dt == WGINFER_DTYPE_F32 ? 4 : 2; }
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// qkv rows [T, (nh + 2 nkvh) * dh] (q/k columns pair-interleaved: column 2i,
// 2i+1 = rotation pair i) -> q_rope [T, nh, dh] and, for the k/v heads, the
// cache of sequence seq(t) at position pos[t]. One thread per rotation pair.
template <typename T>
__global__ void __launch_bounds__(128) qkv_post_kernel(const T *__restrict__ qkv, T *__restrict__ q_out, T *kcache,
                                                       T *vcache, const int64_t *__restrict__ pos,
                                                       const float2 *__restrict__ table, int T_rows, int nh,
                                                       int nkvh, int dh, int maxseq, int prefill_seq,
                                                       size_t seq_stride, unsigned long long *err) {
    const int t = blockIdx.y;
    const int half = dh / 2;
    const int nq = nh + 2 * nkvh;
    int64_t p = pos[t];
    if (p < 0 || p >= maxseq) {
        if (threadIdx.x == 0 && blockIdx.x == 0) record_device_error(err, 3, p);
        return;
    }
    const int seq = prefill_seq >= 0 ? prefill_seq : t;
    const T *row = qkv + (size_t)t * nq * dh;
    T *kc = kcache + (size_t)seq * seq_stride + (size_t)p * nkvh * dh;
    T *vc = vcache + (size_t)seq * seq_stride + (size_t)p * nkvh * dh;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < (nh + nkvh) * half + nkvh * dh;
         idx += gridDim.x * blockDim.x) {
        if (idx < (nh + nkvh) * half) {
            const int h = idx / half, j = idx - h * half;  // h < nh: q head; else k head h - nh
            const float2 cs = table[(size_t)p * half + j];
            // rotation partners sit side by side (pair-interleaved q/k rows)
            const float a = ldf(row, 2 * (size_t)idx), b = ldf(row, 2 * (size_t)idx + 1);
            const float o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
            const float o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
            T *dst = h < nh ? q_out + ((size_t)t * nh + h) * dh : kc + (size_t)(h - nh) * dh;
            stf(dst, j, o0);
            stf(dst, j + half, o1);
        } else {
            const int e = idx - (nh + nkvh) * half;  // v element
            vc[e] = row[(size_t)(nh + nkvh) * dh + e];
        }
    }
}

// act[t, j] = swiglu(gu[t, j], gu[t, di + j]) (swiglu_cpu.cpp:11).
template <typename T, bool kRef>
__global__ void __launch_bounds__(256) swiglu_rows_kernel(T *__restrict__ act, const T *__restrict__ gu, int T_rows,
                                                          int di) {
    const size_t n = (size_t)T_rows * di;
    for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (size_t)gridDim.x * 256) {
        const size_t t = i / di, j = i - t * di;  // gate and up rows are interleaved
        const float g = ldf(gu, t * 2 * di + 2 * j), u = ldf(gu, t * 2 * di + 2 * j + 1);
        const float e = kRef ? expf_glibc(-g) : expf(-g);
        stf(act, i, __fdiv_rn(__fmul_rn(u, g), __fadd_rn(1.0f, e)));
    }
}

// dst row map(r) = src row r for r < nrows; map: kind 0 = rotation-pair
// interleave of heads of dh rows (row h*dh + c -> h*dh + 2*(c % half) + c / half),
// kind 1 = stride 2 from `first` (row r -> 2 r + first).
__global__ void permute_rows_kernel(char *dst, const char *src, int nrows, size_t row_bytes, int kind, int dh,
                                    int first) {
    for (int r = blockIdx.x; r < nrows; r += gridDim.x) {
        int d;
        if (kind == 0) {
            const int h = r / dh, c = r - h * dh, half = dh / 2;
            d = h * dh + 2 * (c % half) + c / half;
        } else {
            d = 2 * r + first;
        }
        const char *s = src + (size_t)r * row_bytes;
        char *o = dst + (size_t)d * row_bytes;
        for (size_t i = threadIdx.x; i < row_bytes; i += blockDim.x) o[i] = s[i];
    }
}

__global__ void fill_positions_kernel(int64_t *pos, int64_t start, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) pos[i] = start + i;
}

}  // namespace
}  // namespace wgb

using namespace wgb;

struct LayerW {
    void *attn_norm, *qkv_w, *qkv_b, *o_w, *mlp_norm, *gu_w, *down_w;
};

struct wgbQwen2Model {
    wgbQwen2Meta m;
    int device = 0, max_batch = 1, chunk = 1;
    wginferDataType_t dt;
    size_t es = 2;
    cudaStream_t stream = nullptr;
    char *arena = nullptr;
    size_t arena_bytes = 0;
    // weights
    void *in_embed, *out_embed, *out_norm;
    std::vector<LayerW> L;
    float2 *rope_table;
    // caches and state
    void *kc, *vc;
    size_t seq_stride;  // elements per sequence per layer in kc / vc
    int64_t *lens, *tokens, *pos;
    // activations (rows = max(max_batch, chunk))
    void *x, *xn, *qkv, *qr, *att, *gu, *act, *logits;
    void *attn_ws;
    unsigned long long *amax_keys;  // [max_batch] fused lm_head + argmax keys (zero between launches)
    unsigned *amax_count;           // its CTA arrival counter (zero between launches)
    size_t attn_ws_bytes;
    int64_t *h_pinned;  // pinned host staging for token ids
    unsigned long long sample_seed = 0, sample_step = 0;  // device sampler: seed, draws so far
    size_t h_pinned_n;
    std::vector<size_t> h_lens;
    std::vector<bool> has_bias;
    // graphs per (batch, numerics)
    std::vector<cudaGraphExec_t> graphs[2];


    size_t nq() const { return (m.nh + 2 * m.nkvh) * m.dh; }
    void *layer_k(size_t l) const { return (char *)kc + l * max_batch * seq_stride * es; }
    void *layer_v(size_t l) const { return (char *)vc + l * max_batch * seq_stride * es; }
};

namespace {

int cuda_err(const char *what) { return check_launch(what); }



// Per-launch device timing of an eagerly launched decode step
// (wgb_qwen2_trace_step): an event after every launch on the model stream.
struct Tracer {
    bool on = false;
    cudaStream_t s = nullptr;
    std::vector<cudaEvent_t> ev;
    std::vector<const char *> names;
    void mark(const char *name) {
        if (!on) return;
        cudaEvent_t e;
        cudaEventCreate(&e);
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(s, &st);
        if (st == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
        else cudaEventRecord(e, s);
        ev.push_back(e);
        names.push_back(name);
    }
};
thread_local Tracer t_trace;
#define WGB_TRACE(name) t_trace.mark(name)

// self_attention for one layer: dense causal over the prefill sequence's
// cache, or batched decode over every row's own cache.
int attention(wgbQwen2Model *M, size_t l, int T, int prefill_seq, size_t total_len, bool ref,
              const void *pf_ptr = nullptr, size_t pf_bytes = 0) {
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    const float scale = 1.0f / sqrtf((float)m.dh);
    if (prefill_seq >= 0) {
        const char *kb = (const char *)M->layer_k(l) + (size_t)prefill_seq * M->seq_stride * M->es;
        const char *vb = (const char *)M->layer_v(l) + (size_t)prefill_seq * M->seq_stride * M->es;
        int prev = wgb_get_numerics();
        wgb_set_numerics(ref ? WGB_NUMERICS_REFERENCE : WGB_NUMERICS_FAST);
        int rc = wgb_self_attention_ex(M->att, M->qr, kb, vb, M->dt, T, m.nh, m.nkvh, m.dh, m.dh, total_len, scale,
                                       M->attn_ws, M->attn_ws_bytes, s);
        wgb_set_numerics(prev);
        return rc;
    }
    return attn_decode(M->dt, M->att, M->qr, M->layer_k(l), M->layer_v(l), M->seq_stride, M->lens, T, (int)m.nh,
                       (int)m.nkvh, (int)m.dh, (int)m.maxseq, scale, M->attn_ws, ref, s, pf_ptr, pf_bytes);
}

// Positions of the layer's rows: the prefill chunk's (filled per chunk), or,
// in batched decode, each sequence's current length (row b's new token sits
// at lens[b]; the step's argmax advances lens once the token is chosen).
const int64_t *positions(const wgbQwen2Model *M, int prefill_seq) { return prefill_seq >= 0 ? M->pos : M->lens; }

// One transformer layer over T rows (model.cpp:243-328), REFERENCE numerics:
// the reference's op sequence with each op in the reference summation order.
int run_layer_ref(wgbQwen2Model *M, size_t l, int T, int prefill_seq, size_t total_len) {
    const bool ref = true;
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    const LayerW &w = M->L[l];
    const int hs = (int)m.hs, di = (int)m.di;
    int rc;
    if ((rc = wgb_rms_norm(M->xn, M->x, w.attn_norm, M->dt, T, hs, m.epsilon, s))) return rc;
    if ((rc = linear_forward(M->dt, M->qkv, M->xn, w.qkv_w, w.qkv_b, nullptr, T, (int)M->nq(), hs, ref, s))) return rc;
    {
        const int half = (int)m.dh / 2;
        const int work = (int)((m.nh + m.nkvh) * half + m.nkvh * m.dh);
        dim3 grid((unsigned)((work + 127) / 128), (unsigned)T);
        WGB_DISPATCH_FLOAT(M->dt, Tt,
            qkv_post_kernel<Tt><<<grid, 128, 0, s>>>((const Tt *)M->qkv, (Tt *)M->qr, (Tt *)M->layer_k(l),
                                                     (Tt *)M->layer_v(l), positions(M, prefill_seq), M->rope_table, T, (int)m.nh,
                                                     (int)m.nkvh, (int)m.dh, (int)m.maxseq, prefill_seq,
                                                     M->seq_stride, dev_error_ptr()));
        if ((rc = cuda_err("qkv_post"))) return rc;
    }
    if ((rc = attention(M, l, T, prefill_seq, total_len, ref))) return rc;
    // o_proj with the residual add fused: x = x + o(att)
    if ((rc = linear_forward(M->dt, M->x, M->att, w.o_w, nullptr, M->x, T, hs, (int)(m.nh * m.dh), ref, s))) return rc;
    if ((rc = wgb_rms_norm(M->xn, M->x, w.mlp_norm, M->dt, T, hs, m.epsilon, s))) return rc;
    if ((rc = linear_forward(M->dt, M->gu, M->xn, w.gu_w, nullptr, nullptr, T, 2 * di, hs, ref, s))) return rc;
    {
        const size_t n = (size_t)T * di;
        const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 8);
        WGB_DISPATCH_FLOAT(M->dt, Tt,
            swiglu_rows_kernel<Tt, true><<<blocks, 256, 0, s>>>((Tt *)M->act, (const Tt *)M->gu, T, di));
        if ((rc = cuda_err("swiglu_rows"))) return rc;
    }
    return linear_forward(M->dt, M->x, M->act, w.down_w, nullptr, M->x, T, hs, di, ref, s);
}


// The same layer in FAST numerics: five launches, each chained to the
// previous one by programmatic dependent launch (decode_gemv.cu).
int run_layer_fast(wgbQwen2Model *M, size_t l, int T, int prefill_seq, size_t total_len) {
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    const LayerW &w = M->L[l];
    const int hs = (int)m.hs, di = (int)m.di, half = (int)m.dh / 2;
    const size_t es = M->es;
    const size_t qkv_b = M->nq() * m.hs * es, o_b = m.hs * m.nh * m.dh * es, gu_b = 2 * m.di * m.hs * es,
                 down_b = m.hs * m.di * es;
    const bool last = l + 1 == m.nlayer;
    const void *next_qkv = last ? M->out_embed : M->L[l + 1].qkv_w;
    const size_t next_qkv_b = last ? std::min<size_t>(m.voc * m.hs * es, 32u << 20) : qkv_b;
    int rc;
    DecodeGemvParams p{};
    p.M0 = T;
    p.pf_ptr[0] = w.o_w;      // each kernel pulls the following weights into L2
    p.pf_bytes[0] = o_b;
    p.pf_ptr[1] = w.gu_w;
    p.pf_bytes[1] = gu_b / 2;
    p.eps = m.epsilon;
    p.err = dev_error_ptr();
    // rms_norm + q/k/v projection + bias + RoPE + K/V cache append
    p.w = w.qkv_w;
    p.x = M->x;
    p.N = (int)M->nq();
    p.K = hs;
    p.groups = (int)((m.nh + m.nkvh) * half + m.nkvh * m.dh / 2);
    p.norm_w = w.attn_norm;
    p.bias = w.qkv_b;
    p.pos = positions(M, prefill_seq);
    p.table = M->rope_table;
    p.q_out = M->qr;
    p.kc = M->layer_k(l);
    p.vc = M->layer_v(l);
    p.seq_stride = M->seq_stride;
    p.nh = (int)m.nh;
    p.nkvh = (int)m.nkvh;
    p.dh = (int)m.dh;
    p.maxseq = (int)m.maxseq;
    p.prefill_seq = prefill_seq;
    p.xn = M->xn;
    if ((rc = decode_gemv(M->dt, p, DG_PRO_RMS, DG_EPI_ROPEKV, s))) return rc;
    WGB_TRACE("qkv_gemv+rms+rope+kv");
    // no L2 prefetch from attention: its own K/V reads are latency-critical
    if ((rc = attention(M, l, T, prefill_seq, total_len, false))) return rc;
    WGB_TRACE("attention");
    // o_proj + residual
    DecodeGemvParams o{};
    o.M0 = T;
    o.w = w.o_w;
    o.x = M->att;
    o.N = hs;
    o.K = (int)(m.nh * m.dh);
    o.groups = (hs + 1) / 2;
    o.out = M->x;
    o.ldo = hs;
    o.res = M->x;
    o.pf_ptr[0] = w.down_w;
    o.pf_bytes[0] = down_b;
    if ((rc = decode_gemv(M->dt, o, DG_PRO_PLAIN, DG_EPI_STORE, s))) return rc;
    WGB_TRACE("o_gemv+residual");
    // rms_norm + gate/up projection + SwiGLU
    DecodeGemvParams g{};
    g.M0 = T;
    g.w = w.gu_w;
    g.x = M->x;
    g.N = 2 * di;
    g.K = hs;
    g.groups = di;
    g.norm_w = w.mlp_norm;
    g.eps = m.epsilon;
    g.out = M->act;
    g.ldo = di;
    g.di = di;
    g.pf_ptr[0] = next_qkv;
    g.pf_bytes[0] = next_qkv_b;
    g.xn = M->xn;
    if ((rc = decode_gemv(M->dt, g, DG_PRO_RMS, DG_EPI_SWIGLU, s))) return rc;
    WGB_TRACE("gate_up_gemv+rms+swiglu");
    // down_proj + residual
    DecodeGemvParams d{};
    d.M0 = T;
    d.w = w.down_w;
    d.x = M->act;
    d.N = hs;
    d.K = di;
    d.groups = (hs + 1) / 2;
    d.out = M->x;
    d.ldo = hs;
    d.res = M->x;
    if (!last) {
        d.pf_ptr[0] = M->L[l + 1].o_w;
        d.pf_bytes[0] = o_b;
        d.pf_ptr[1] = M->L[l + 1].gu_w;
        d.pf_bytes[1] = gu_b / 2;
    } else {
        d.pf_ptr[0] = (const char *)M->out_embed + next_qkv_b;
        d.pf_bytes[0] = std::min<size_t>(m.voc * m.hs * es - next_qkv_b, 32u << 20);
    }
    rc = decode_gemv(M->dt, d, DG_PRO_PLAIN, DG_EPI_STORE, s);
    WGB_TRACE("down_gemv+residual");
    return rc;
}

// Whether a decode step of B sequences takes the REFERENCE chain kernels
// (ref_decode.cu): up to kRefChainMaxM rows, caches the decode attention holds.
bool ref_decode_fast_ok(const wgbQwen2Model *M, int B) {
    const wgbQwen2Meta &m = M->m;
    if (B > kRefChainMaxM) return false;
    if (!ref_attn_decode_ok(M->dt, (int)m.nh, (int)m.nkvh, (int)m.dh, (int)m.maxseq, M->kc, M->vc, M->seq_stride))
        return false;
    DecodeGemvParams p{};
    p.M0 = B;
    p.w = M->L[0].down_w;
    p.x = M->act;
    p.N = (int)m.hs;
    p.K = (int)m.di;  // the longest rows; the other projections have K = hs or nh * dh
    if (!ref_chain_ok(M->dt, p)) return false;
    p.K = (int)m.hs;
    if (!ref_chain_ok(M->dt, p)) return false;
    p.K = (int)(m.nh * m.dh);
    return ref_chain_ok(M->dt, p);
}

// One decode layer for B <= kRefChainMaxM sequences in REFERENCE numerics:
// the op sequence of run_layer_ref (model.cpp:243-328) in five launches
// chained by programmatic dependent launch, every sum in the reference's
// order (ref_decode.cu): rms_norm + q/k/v + bias + RoPE + K/V append;
// attention; o + residual; rms_norm + gate/up + SwiGLU; down + residual.
int run_layer_ref_decode(wgbQwen2Model *M, size_t l, int B) {
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    const LayerW &w = M->L[l];
    const int hs = (int)m.hs, di = (int)m.di;
    int rc;
    DecodeGemvParams p{};
    p.M0 = B;
    p.err = dev_error_ptr();
    p.eps = m.epsilon;
    p.w = w.qkv_w;
    p.x = M->x;
    p.N = (int)M->nq();
    p.K = hs;
    p.norm_w = w.attn_norm;
    p.bias = w.qkv_b;
    p.pos = M->lens;
    p.table = M->rope_table;
    p.q_out = M->qr;
    p.kc = M->layer_k(l);
    p.vc = M->layer_v(l);
    p.seq_stride = M->seq_stride;
    p.nh = (int)m.nh;
    p.nkvh = (int)m.nkvh;
    p.dh = (int)m.dh;
    p.maxseq = (int)m.maxseq;
    p.prefill_seq = -1;
    if ((rc = ref_chain_gemv(M->dt, p, DG_PRO_RMS, DG_EPI_ROPEKV, s))) return rc;
    WGB_TRACE("ref qkv+rms+rope+kv");
    if ((rc = ref_attn_decode(M->dt, M->att, M->qr, M->layer_k(l), M->layer_v(l), M->seq_stride, M->lens, B,
                              (int)m.nh, (int)m.nkvh, (int)m.dh, (int)m.maxseq, 1.0f / sqrtf((float)m.dh), s)))
        return rc;
    WGB_TRACE("ref attention");
    DecodeGemvParams o{};
    o.M0 = B;
    o.err = p.err;
    o.w = w.o_w;
    o.x = M->att;
    o.N = hs;
    o.K = (int)(m.nh * m.dh);
    o.out = M->x;
    o.ldo = hs;
    o.res = M->x;
    if ((rc = ref_chain_gemv(M->dt, o, DG_PRO_PLAIN, DG_EPI_STORE, s))) return rc;
    WGB_TRACE("ref o+residual");
    DecodeGemvParams g{};
    g.M0 = B;
    g.err = p.err;
    g.w = w.gu_w;
    g.x = M->x;
    g.N = 2 * di;
    g.K = hs;
    g.norm_w = w.mlp_norm;
    g.eps = m.epsilon;
    g.out = M->act;
    g.ldo = di;
    if ((rc = ref_chain_gemv(M->dt, g, DG_PRO_RMS, DG_EPI_SWIGLU, s))) return rc;
    WGB_TRACE("ref gate_up+rms+swiglu");
    DecodeGemvParams d{};
    d.M0 = B;
    d.err = p.err;
    d.w = w.down_w;
    d.x = M->act;
    d.N = hs;
    d.K = di;
    d.out = M->x;
    d.ldo = hs;
    d.res = M->x;
    rc = ref_chain_gemv(M->dt, d, DG_PRO_PLAIN, DG_EPI_STORE, s);
    WGB_TRACE("ref down+residual");
    return rc;
}

int run_layer(wgbQwen2Model *M, size_t l, int T, int prefill_seq, size_t total_len, bool ref) {
    return ref ? run_layer_ref(M, l, T, prefill_seq, total_len) : run_layer_fast(M, l, T, prefill_seq, total_len);
}

// final rms_norm + lm_head for `rows` rows of x starting at x_row, into logits.
int lm_head(wgbQwen2Model *M, const void *x_row, int rows, void *logits, bool ref) {
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    int rc;
    if (ref) {
        if ((rc = wgb_rms_norm(M->xn, x_row, M->out_norm, M->dt, rows, m.hs, m.epsilon, s))) return rc;
        return linear_forward(M->dt, logits, M->xn, M->out_embed, nullptr, nullptr, rows, (int)m.voc, (int)m.hs, ref, s);
    }
    DecodeGemvParams p{};
    p.M0 = rows;
    p.w = M->out_embed;
    p.x = x_row;
    p.N = (int)m.voc;
    p.K = (int)m.hs;
    p.groups = (int)(m.voc + 1) / 2;
    p.norm_w = M->out_norm;
    p.eps = m.epsilon;
    p.out = logits;
    p.ldo = (int)m.voc;
    p.xn = M->xn;
    return decode_gemv(M->dt, p, DG_PRO_RMS, DG_EPI_STORE, s);
}

// Decode step body for sequences [0, B) (captured into a graph).
int decode_body(wgbQwen2Model *M, int B, bool ref) {
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    int rc;

    if ((rc = wgb_embedding(M->x, M->tokens, M->in_embed, M->dt, B, m.hs, m.voc, s))) return rc;
    WGB_TRACE("embedding");
    if (ref && ref_decode_fast_ok(M, B)) {
        for (size_t l = 0; l < m.nlayer; l++)
            if ((rc = run_layer_ref_decode(M, l, B))) return rc;
        // final rms_norm + lm_head + greedy argmax + lengths advanced, one launch
        DecodeGemvParams p{};
        p.M0 = B;
        p.err = dev_error_ptr();
        p.w = M->out_embed;
        p.x = M->x;
        p.N = (int)m.voc;
        p.K = (int)m.hs;
        p.norm_w = M->out_norm;
        p.eps = m.epsilon;
        p.out = M->logits;
        p.ldo = (int)m.voc;
        p.amax_keys = M->amax_keys;
        p.amax_count = M->amax_count;
        p.tokens = M->tokens;
        p.lens = M->lens;
        p.maxlen = (int64_t)m.maxseq;
        rc = ref_chain_gemv(M->dt, p, DG_PRO_RMS, DG_EPI_ARGMAX, s);
        WGB_TRACE("ref lm_head+rms+argmax+advance");
        return rc;
    }
    for (size_t l = 0; l < m.nlayer; l++)
        if ((rc = run_layer(M, l, B, -1, 0, ref))) return rc;
    if (!ref && (B <= 8 || (M->dt == WGINFER_DTYPE_BF16 && B <= 256))) {
        // final rms_norm + lm_head + greedy argmax + lengths advanced: one
        // launch up to 8 rows (GEMV), else rms_norm + the tensor-core GEMM
        // with the argmax epilogue
        DecodeGemvParams p{};
        p.M0 = B;
        p.err = dev_error_ptr();
        p.w = M->out_embed;
        p.x = M->x;
        p.N = (int)m.voc;
        p.K = (int)m.hs;
        p.groups = (int)(m.voc + 1) / 2;
        p.norm_w = M->out_norm;
        p.eps = m.epsilon;
        p.out = M->logits;
        p.ldo = (int)m.voc;
        p.xn = M->xn;
        p.amax_keys = M->amax_keys;
        p.amax_count = M->amax_count;
        p.tokens = M->tokens;
        p.lens = M->lens;
        p.maxlen = (int64_t)m.maxseq;
        rc = decode_gemv(M->dt, p, DG_PRO_RMS, DG_EPI_ARGMAX, s);
        WGB_TRACE("lm_head_gemv+rms+argmax+advance");
        return rc;
    }
    if ((rc = lm_head(M, M->x, B, M->logits, ref))) return rc;
    WGB_TRACE("lm_head_gemv+rms");
    // the greedy tokens, and every sequence one position longer
    if ((rc = argmax_rows_advance(M->tokens, M->logits, M->dt, B, m.voc, M->lens, (int64_t)m.maxseq, s))) return rc;
    WGB_TRACE("argmax+advance");
    return WGB_OK;
}

int prefill_impl(wgbQwen2Model *M, int seq, const int64_t *ids_host, size_t n, bool ref) {
    const wgbQwen2Meta &m = M->m;
    cudaStream_t s = M->stream;
    size_t cache_len = M->h_lens[seq];
    WGB_REQUIRE(cache_len + n <= m.maxseq, WGB_ERR_OUT_OF_RANGE, "prefill: %zu + %zu tokens exceed maxseq %zu", cache_len,
                n, (size_t)m.maxseq);
    int rc;
    for (size_t off = 0; off < n; off += M->chunk) {
        const int T = (int)std::min<size_t>(M->chunk, n - off);
        if (M->h_pinned_n < (size_t)T) return set_error(WGB_ERR_INVALID_ARGUMENT, "staging too small");
        // stage ids through pinned memory; the copy must finish before the buffer is reused
        if (cudaStreamSynchronize(s) != cudaSuccess) return cuda_err("prefill sync");
        memcpy(M->h_pinned, ids_host + off, (size_t)T * sizeof(int64_t));
        int64_t *ids_dev = M->pos + M->chunk;  // second half of the position buffer holds ids
        if (cudaMemcpyAsync(ids_dev, M->h_pinned, (size_t)T * sizeof(int64_t), cudaMemcpyHostToDevice, s) != cudaSuccess)
            return cuda_err("prefill H2D");
        fill_positions_kernel<<<(T + 255) / 256, 256, 0, s>>>(M->pos, (int64_t)cache_len, T);
        if ((rc = wgb_embedding(M->x, ids_dev, M->in_embed, M->dt, T, m.hs, m.voc, s))) return rc;
        const size_t total = cache_len + T;
        for (size_t l = 0; l < m.nlayer; l++)
            if ((rc = run_layer(M, l, T, seq, total, ref))) return rc;
        cache_len = total;
        if (off + T == n) {
            const char *last = (const char *)M->x + (size_t)(T - 1) * m.hs * M->es;
            void *lg = (char *)M->logits + (size_t)seq * m.voc * M->es;
            if ((rc = lm_head(M, last, 1, lg, ref))) return rc;
            if ((rc = wgb_argmax_rows(M->tokens + seq, nullptr, lg, M->dt, 1, m.voc, s))) return rc;
        }
    }
    M->h_lens[seq] = cache_len;
    int64_t l64 = (int64_t)cache_len;
    if (cudaMemcpyAsync(M->lens + seq, &l64, sizeof(int64_t), cudaMemcpyHostToDevice, s) != cudaSuccess)
        return cuda_err("prefill lens");
    if (cudaStreamSynchronize(s) != cudaSuccess) return cuda_err("prefill");
    return WGB_OK;
}

int get_graph(wgbQwen2Model *M, int B, bool ref, cudaGraphExec_t *out) {
    auto &g = M->graphs[ref ? 1 : 0];
    if (g.size() < (size_t)M->max_batch + 1) g.resize(M->max_batch + 1, nullptr);
    if (g[B]) {
        *out = g[B];
        return WGB_OK;
    }
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(M->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return cuda_err("begin capture");
    int rc = decode_body(M, B, ref);
    cudaError_t e = cudaStreamEndCapture(M->stream, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (e != cudaSuccess) return cuda_err("end capture");
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_err("graph instantiate");
    g[B] = exec;
    *out = exec;
    return WGB_OK;
}

// Host table with the reference's exact expressions (rope_cpu.cpp:13-36).
std::vector<float2> build_rope_table(size_t maxseq, size_t dh, float theta) {
    const size_t half = dh / 2;
    std::vector<float> denom(half);
    for (size_t j = 0; j < half; ++j) denom[j] = ::powf(theta, (2.0f * (float)j) / (float)dh);
    std::vector<float2> t(maxseq * half);
    for (size_t p = 0; p < maxseq; ++p) {
        const float pf = (float)(int64_t)p;
        for (size_t j = 0; j < half; ++j) {
            const float phi = pf / denom[j];
            t[p * half + j] = make_float2(::cosf(phi), ::sinf(phi));
        }
    }
    return t;
}

}  // namespace

extern "C" {

int wgb_qwen2_create(const wgbQwen2Meta *meta, int device, int max_batch, wgbQwen2Model **out) {
    WGB_REQUIRE(meta && out, WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_create: null argument");
    WGB_REQUIRE(meta->dtype == WGINFER_DTYPE_BF16 || meta->dtype == WGINFER_DTYPE_F32 || meta->dtype == WGINFER_DTYPE_F16,
                WGB_ERR_UNSUPPORTED_DTYPE, "wgb_qwen2_create: dtype %d", meta->dtype);
    WGB_REQUIRE(meta->nlayer > 0 && meta->hs > 0 && meta->nh > 0 && meta->nkvh > 0 && meta->nh % meta->nkvh == 0 &&
                    meta->dh > 0 && meta->dh % 2 == 0 && meta->di > 0 && meta->maxseq > 0 && meta->voc > 0,
                WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_create: bad meta");
    WGB_REQUIRE(max_batch >= 1 && max_batch <= 4096, WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_create: max_batch %d", max_batch);
    if (cudaSetDevice(device) != cudaSuccess) return cuda_err("wgb_qwen2_create: cudaSetDevice");
    auto *M = new wgbQwen2Model();
    M->m = *meta;
    M->device = device;
    M->max_batch = max_batch;
    M->dt = (wginferDataType_t)meta->dtype;
    M->es = dsize(meta->dtype);
    M->chunk = (int)std::min<size_t>(meta->maxseq, 2048);
    const wgbQwen2Meta &m = M->m;
    const size_t es = M->es, rows = std::max<size_t>(max_batch, M->chunk);
    M->seq_stride = m.maxseq * m.nkvh * m.dh;
    const bool ref_ws = true;  // size the workspace for either numerics mode
    const size_t ws_dec = std::max(attn_decode_workspace(max_batch, (int)m.nh, (int)m.nkvh, (int)m.dh, (int)m.maxseq, false),
                                   attn_decode_workspace(max_batch, (int)m.nh, (int)m.nkvh, (int)m.dh, (int)m.maxseq, ref_ws));
    int prev = wgb_get_numerics();
    wgb_set_numerics(WGB_NUMERICS_FAST);
    size_t ws_pre = wgb_self_attention_workspace_size(M->chunk, m.nh, m.nkvh, m.dh, m.dh, m.maxseq);
    wgb_set_numerics(WGB_NUMERICS_REFERENCE);
    ws_pre = std::max(ws_pre, wgb_self_attention_workspace_size(M->chunk, m.nh, m.nkvh, m.dh, m.dh, m.maxseq));
    wgb_set_numerics(prev);
    M->attn_ws_bytes = std::max<size_t>(std::max(ws_dec, ws_pre), 256);

    // arena plan
    struct Item { void **p; size_t bytes; };
    std::vector<Item> items;
    M->L.resize(m.nlayer);
    items.push_back({&M->in_embed, m.voc * m.hs * es});
    items.push_back({&M->out_embed, m.voc * m.hs * es});
    items.push_back({&M->out_norm, m.hs * es});
    for (size_t l = 0; l < m.nlayer; l++) {
        LayerW &w = M->L[l];
        items.push_back({&w.attn_norm, m.hs * es});
        items.push_back({&w.qkv_w, M->nq() * m.hs * es});
        items.push_back({&w.qkv_b, M->nq() * es});
        items.push_back({&w.o_w, m.hs * m.nh * m.dh * es});
        items.push_back({&w.mlp_norm, m.hs * es});
        items.push_back({&w.gu_w, 2 * m.di * m.hs * es});
        items.push_back({&w.down_w, m.hs * m.di * es});
    }
    items.push_back({(void **)&M->rope_table, m.maxseq * (m.dh / 2) * sizeof(float2)});
    items.push_back({&M->kc, m.nlayer * (size_t)max_batch * M->seq_stride * es});
    items.push_back({&M->vc, m.nlayer * (size_t)max_batch * M->seq_stride * es});
    items.push_back({(void **)&M->lens, (size_t)max_batch * 8});
    items.push_back({(void **)&M->tokens, (size_t)max_batch * 8});
    items.push_back({(void **)&M->pos, 2 * rows * 8});
    items.push_back({&M->x, rows * m.hs * es});
    items.push_back({&M->xn, rows * m.hs * es});
    items.push_back({&M->qkv, rows * M->nq() * es});
    items.push_back({&M->qr, rows * m.nh * m.dh * es});
    items.push_back({&M->att, rows * m.nh * m.dh * es});
    items.push_back({&M->gu, rows * 2 * m.di * es});
    items.push_back({&M->act, rows * m.di * es});
    items.push_back({&M->logits, (size_t)max_batch * m.voc * es});
    items.push_back({&M->attn_ws, M->attn_ws_bytes});
    items.push_back({(void **)&M->amax_keys, (size_t)max_batch * sizeof(unsigned long long)});
    items.push_back({(void **)&M->amax_count, sizeof(unsigned)});

    size_t total = 0;
    for (auto &it : items) total += align256(it.bytes);
    if (cudaMalloc((void **)&M->arena, total) != cudaSuccess) {
        cudaGetLastError();
        delete M;
        return set_error(WGB_ERR_NO_MEMORY, "wgb_qwen2_create: arena of %zu bytes", total);
    }
    M->arena_bytes = total;
    size_t off = 0;
    for (auto &it : items) {
        *it.p = M->arena + off;
        off += align256(it.bytes);
    }
    int rc = WGB_OK;
    if (cudaStreamCreateWithFlags(&M->stream, cudaStreamNonBlocking) != cudaSuccess) rc = cuda_err("stream");
    // like the reference's sampler (model.cpp:131), seeded from the system's
    // random device: draws differ between models and runs
    M->sample_seed = ((unsigned long long)std::random_device{}() << 32) ^ std::random_device{}();
    // zero everything (biases default to zero, like the reference's dummy biases)
    if (!rc && cudaMemsetAsync(M->arena, 0, total, M->stream) != cudaSuccess) rc = cuda_err("arena memset");
    auto table = build_rope_table(m.maxseq, m.dh, m.theta);
    if (!rc && cudaMemcpyAsync(M->rope_table, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice,
                               M->stream) != cudaSuccess)
        rc = cuda_err("rope table");
    M->h_pinned_n = (size_t)M->chunk;
    if (!rc && cudaMallocHost((void **)&M->h_pinned, M->h_pinned_n * sizeof(int64_t)) != cudaSuccess)
        rc = cuda_err("pinned staging");
    if (!rc && cudaStreamSynchronize(M->stream) != cudaSuccess) rc = cuda_err("create sync");
    attn_prepare();
    decode_gemv_prepare();
    ref_decode_prepare();

    dev_error_ptr();  // resolve the error-word address outside any graph capture
    M->h_lens.assign(max_batch, 0);
    if (rc) {
        wgb_qwen2_destroy(M);
        return rc;
    }
    *out = M;
    return WGB_OK;
}

int wgb_qwen2_destroy(wgbQwen2Model *M) {
    if (!M) return WGB_OK;
    cudaSetDevice(M->device);
    if (M->stream) cudaStreamSynchronize(M->stream);
    for (auto &g : M->graphs)
        for (auto e : g)
            if (e) cudaGraphExecDestroy(e);
    if (M->h_pinned) cudaFreeHost(M->h_pinned);
    if (M->arena) cudaFree(M->arena);
    if (M->stream) cudaStreamDestroy(M->stream);
    delete M;
    return WGB_OK;
}

int wgb_qwen2_set_weight(wgbQwen2Model *M, const char *name, int layer, const void *src, size_t bytes, int on_host) {
    WGB_REQUIRE(M && name && src, WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_set_weight: null argument");
    const wgbQwen2Meta &m = M->m;
    const size_t es = M->es;
    std::string n(name);
    void *dst = nullptr;
    size_t want = 0, row_bytes = 0, nrows = 0;
    int kind = -1, first = 0;
    if (layer < 0) {
        if (n == "in_embed") dst = M->in_embed, want = m.voc * m.hs * es;
        else if (n == "out_embed") dst = M->out_embed, want = m.voc * m.hs * es;
        else if (n == "out_norm_w") dst = M->out_norm, want = m.hs * es;
    } else {
        WGB_REQUIRE((size_t)layer < m.nlayer, WGB_ERR_OUT_OF_RANGE, "layer %d out of range", layer);
        LayerW &w = M->L[layer];
        const size_t qn = m.nh * m.dh, kn = m.nkvh * m.dh;
        // q/k rows are stored rotation-pair interleaved, gate/up rows
        // interleaved (see decode_common.cuh); `kind` selects the row map
        if (n == "attn_norm_w") dst = w.attn_norm, want = m.hs * es;
        else if (n == "attn_q_w") dst = w.qkv_w, want = qn * m.hs * es, kind = 0, row_bytes = m.hs * es, nrows = qn;
        else if (n == "attn_k_w")
            dst = (char *)w.qkv_w + qn * m.hs * es, want = kn * m.hs * es, kind = 0, row_bytes = m.hs * es, nrows = kn;
        else if (n == "attn_v_w") dst = (char *)w.qkv_w + (qn + kn) * m.hs * es, want = kn * m.hs * es;
        else if (n == "attn_q_b") dst = w.qkv_b, want = qn * es, kind = 0, row_bytes = es, nrows = qn;
        else if (n == "attn_k_b") dst = (char *)w.qkv_b + qn * es, want = kn * es, kind = 0, row_bytes = es, nrows = kn;
        else if (n == "attn_v_b") dst = (char *)w.qkv_b + (qn + kn) * es, want = kn * es;
        else if (n == "attn_o_w") dst = w.o_w, want = m.hs * qn * es;
        else if (n == "mlp_norm_w") dst = w.mlp_norm, want = m.hs * es;
        else if (n == "mlp_gate_w") dst = w.gu_w, want = m.di * m.hs * es, kind = 1, first = 0, row_bytes = m.hs * es, nrows = m.di;
        else if (n == "mlp_up_w") dst = w.gu_w, want = m.di * m.hs * es, kind = 1, first = 1, row_bytes = m.hs * es, nrows = m.di;
        else if (n == "mlp_down_w") dst = w.down_w, want = m.hs * m.di * es;
    }
    WGB_REQUIRE(dst != nullptr, WGB_ERR_INVALID_ARGUMENT, "unknown Qwen2 weight: %s", name);
    WGB_REQUIRE(bytes == want, WGB_ERR_INVALID_ARGUMENT, "weight %s: %zu bytes given, %zu expected", name, bytes, want);
    cudaSetDevice(M->device);
    if (kind < 0) {
        if (cudaMemcpyAsync(dst, src, bytes, on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, M->stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(M->stream) != cudaSuccess)
            return cuda_err("wgb_qwen2_set_weight");
        return WGB_OK;
    }
    // rows are scattered into the interleaved layout (a one-time copy)
    const void *dsrc = src;
    void *tmp = nullptr;
    if (on_host) {
        if (cudaMalloc(&tmp, bytes) != cudaSuccess) {
            cudaGetLastError();
            return set_error(WGB_ERR_NO_MEMORY, "wgb_qwen2_set_weight: staging %zu bytes", bytes);
        }
        if (cudaMemcpyAsync(tmp, src, bytes, cudaMemcpyHostToDevice, M->stream) != cudaSuccess) {
            cudaFree(tmp);
            return cuda_err("wgb_qwen2_set_weight H2D");
        }
        dsrc = tmp;
    }
    permute_rows_kernel<<<(unsigned)std::min<size_t>(nrows, 4096), 128, 0, M->stream>>>(
        (char *)dst, (const char *)dsrc, (int)nrows, row_bytes, kind, (int)m.dh, first);
    int rc = cuda_err("permute_rows");
    if (cudaStreamSynchronize(M->stream) != cudaSuccess && !rc) rc = cuda_err("wgb_qwen2_set_weight");
    if (tmp) cudaFree(tmp);
    return rc;
}

int wgb_qwen2_reset_cache(wgbQwen2Model *M) {
    WGB_REQUIRE(M, WGB_ERR_INVALID_ARGUMENT, "null model");
    cudaSetDevice(M->device);
    std::fill(M->h_lens.begin(), M->h_lens.end(), 0);
    if (cudaMemsetAsync(M->lens, 0, (size_t)M->max_batch * 8, M->stream) != cudaSuccess ||
        cudaStreamSynchronize(M->stream) != cudaSuccess)
        return cuda_err("reset_cache");
    return WGB_OK;
}

int wgb_qwen2_prefill(wgbQwen2Model *M, int seq, const int64_t *ids, size_t n) {
    WGB_REQUIRE(M && ids && n > 0, WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_prefill: bad argument");
    WGB_REQUIRE(seq >= 0 && seq < M->max_batch, WGB_ERR_OUT_OF_RANGE, "sequence %d", seq);
    cudaSetDevice(M->device);
    return prefill_impl(M, seq, ids, n, wgb_get_numerics() == WGB_NUMERICS_REFERENCE);
}

int wgb_qwen2_decode_step(wgbQwen2Model *M, int B) {
    WGB_REQUIRE(M && B >= 1 && B <= M->max_batch, WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_decode_step: batch %d", B);
    cudaSetDevice(M->device);
    for (int b = 0; b < B; b++)
        WGB_REQUIRE(M->h_lens[b] < M->m.maxseq, WGB_ERR_OUT_OF_RANGE, "sequence %d is full (%zu)", b,
                    (size_t)M->m.maxseq);
    cudaGraphExec_t g;
    int rc = get_graph(M, B, wgb_get_numerics() == WGB_NUMERICS_REFERENCE, &g);
    if (rc) return rc;
    if (cudaGraphLaunch(g, M->stream) != cudaSuccess) return cuda_err("graph launch");
    for (int b = 0; b < B; b++) M->h_lens[b]++;
    return WGB_OK;
}

int wgb_qwen2_infer(wgbQwen2Model *M, const int64_t *ids, size_t n, int top_k, float top_p, float temperature,
                    int64_t *next) {
    WGB_REQUIRE(M && ids && n > 0 && next, WGB_ERR_INVALID_ARGUMENT, "wgb_qwen2_infer: bad argument");
    cudaSetDevice(M->device);
    const bool ref = wgb_get_numerics() == WGB_NUMERICS_REFERENCE;
    int rc;
    if (n == 1) {
        WGB_REQUIRE(M->h_lens[0] < M->m.maxseq, WGB_ERR_OUT_OF_RANGE, "sequence 0 is full");
        M->h_pinned[0] = ids[0];
        if (cudaMemcpyAsync(M->tokens, M->h_pinned, sizeof(int64_t), cudaMemcpyHostToDevice, M->stream) != cudaSuccess)
            return cuda_err("infer H2D");
        if ((rc = wgb_qwen2_decode_step(M, 1))) return rc;
    } else {
        if ((rc = prefill_impl(M, 0, ids, n, ref))) return rc;
    }
    const bool greedy = top_k == 1 && top_p >= 1.0f && std::fabs(temperature - 1.0f) < 1e-6f;
    if (greedy) {
        if (cudaMemcpyAsync(M->h_pinned, M->tokens, sizeof(int64_t), cudaMemcpyDeviceToHost, M->stream) != cudaSuccess ||
            cudaStreamSynchronize(M->stream) != cudaSuccess)
            return cuda_err("infer D2H");
        *next = M->h_pinned[0];
        return WGB_OK;
    }
    // sampling (model.cpp:60-137) on the device: the logits stay there, only
    // the drawn token comes back
    if ((rc = wgb_sample_rows(M->tokens, M->logits, M->dt, 1, M->m.voc, top_k, top_p, temperature, M->sample_seed,
                              M->sample_step++, M->stream)))
        return rc;
    if (cudaMemcpyAsync(M->h_pinned, M->tokens, sizeof(int64_t), cudaMemcpyDeviceToHost, M->stream) != cudaSuccess ||
        cudaStreamSynchronize(M->stream) != cudaSuccess)
        return cuda_err("infer D2H");
    *next = M->h_pinned[0];
    return WGB_OK;
}

int wgb_qwen2_trace_step(wgbQwen2Model *M, int B, int max_launches, float *us, char *names, size_t names_cap,
                         int *n_launches) {
    WGB_REQUIRE(M && us && names && n_launches && B >= 1 && B <= M->max_batch, WGB_ERR_INVALID_ARGUMENT,
                "wgb_qwen2_trace_step: bad argument");
    cudaSetDevice(M->device);
    for (int b = 0; b < B; b++)
        WGB_REQUIRE(M->h_lens[b] < M->m.maxseq, WGB_ERR_OUT_OF_RANGE, "sequence %d is full", b);
    const bool ref = wgb_get_numerics() == WGB_NUMERICS_REFERENCE;
    Tracer &t = t_trace;
    t = Tracer();
    t.on = true;
    t.s = M->stream;
    // capture the step with an event node after every launch, then replay it:
    // per-launch device times without host launch gaps
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int rc = WGB_OK;
    if (cudaStreamBeginCapture(M->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) rc = cuda_err("trace capture");
    if (!rc) {
        t.mark("start");
        rc = decode_body(M, B, ref);
        if (cudaStreamEndCapture(M->stream, &graph) != cudaSuccess && !rc) rc = cuda_err("trace end capture");
    }
    t.on = false;
    if (!rc && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) rc = cuda_err("trace instantiate");
    if (!rc && cudaGraphLaunch(exec, M->stream) != cudaSuccess) rc = cuda_err("trace launch");
    if (cudaStreamSynchronize(M->stream) != cudaSuccess && !rc) rc = cuda_err("trace sync");
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    int n = 0;
    size_t off = 0;
    for (size_t i = 1; i < t.ev.size() && n < max_launches; i++, n++) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, t.ev[i - 1], t.ev[i]);
        us[n] = ms * 1000.f;
        const size_t len = strlen(t.names[i]);
        if (off + len + 2 < names_cap) {
            memcpy(names + off, t.names[i], len);
            off += len;
            names[off++] = '\n';
            names[off] = 0;
        }
    }
    for (auto e : t.ev) cudaEventDestroy(e);
    t = Tracer();
    *n_launches = n;
    if (!rc)
        for (int b = 0; b < B; b++) M->h_lens[b]++;
    return rc;
}

int64_t *wgb_qwen2_token_buffer(wgbQwen2Model *M) { return M ? M->tokens : nullptr; }
wginferStream_t wgb_qwen2_stream(wgbQwen2Model *M) { return M ? (wginferStream_t)M->stream : nullptr; }
size_t wgb_qwen2_cache_len(wgbQwen2Model *M, int seq) {
    return (M && seq >= 0 && seq < M->max_batch) ? M->h_lens[seq] : 0;
}
const void *wgb_qwen2_logits(wgbQwen2Model *M, int seq) {
    return (M && seq >= 0 && seq < M->max_batch) ? (const char *)M->logits + (size_t)seq * M->m.voc * M->es : nullptr;
}

int wgb_qwen2_read_tokens(wgbQwen2Model *M, int64_t *host, int batch) {
    WGB_REQUIRE(M && host && batch >= 1 && batch <= M->max_batch, WGB_ERR_INVALID_ARGUMENT, "read_tokens");
    cudaSetDevice(M->device);
    if (cudaMemcpyAsync(host, M->tokens, (size_t)batch * 8, cudaMemcpyDeviceToHost, M->stream) != cudaSuccess ||
        cudaStreamSynchronize(M->stream) != cudaSuccess)
        return cuda_err("read_tokens");
    return WGB_OK;
}

int wgb_qwen2_read_logits(wgbQwen2Model *M, int seq, float *host) {
    WGB_REQUIRE(M && host && seq >= 0 && seq < M->max_batch, WGB_ERR_INVALID_ARGUMENT, "read_logits");
    cudaSetDevice(M->device);
    const size_t V = M->m.voc;
    const char *src = (const char *)M->logits + (size_t)seq * V * M->es;
    if (M->dt == WGINFER_DTYPE_F32) {
        if (cudaMemcpyAsync(host, src, V * 4, cudaMemcpyDeviceToHost, M->stream) != cudaSuccess ||
            cudaStreamSynchronize(M->stream) != cudaSuccess)
            return cuda_err("read_logits");
        return WGB_OK;
    }
    std::vector<uint16_t> h(V);
    if (cudaMemcpyAsync(h.data(), src, V * 2, cudaMemcpyDeviceToHost, M->stream) != cudaSuccess ||
        cudaStreamSynchronize(M->stream) != cudaSuccess)
        return cuda_err("read_logits");
    for (size_t i = 0; i < V; i++) {
        if (M->dt == WGINFER_DTYPE_BF16) {
            uint32_t u = (uint32_t)h[i] << 16;
            memcpy(&host[i], &u, 4);
        } else {
            __half_raw r;
            r.x = h[i];
            host[i] = __half2float(__half(r));
        }
    }
    return WGB_OK;
}

}  // extern "C"
