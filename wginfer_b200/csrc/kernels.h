// Internal entry points shared between translation units (not exported).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "wginfer_b200.h"

namespace wgb {

// Greedy step of batched decode (argmax.cu): tokens[r] = argmax of logits row
// r, then lens[r] += 1 (up to maxlen), in one launch.
int argmax_rows_advance(int64_t *tokens, const void *logits, wginferDataType_t dtype, size_t rows, size_t numel,
                        int64_t *lens, int64_t maxlen, cudaStream_t s);

// tcgen05 GEMM (linear_tc.cu): true when the tensor-core path takes this call.
bool linear_tc_supported(size_t M, size_t N, size_t K, const void *out, const void *x, const void *w);
int linear_tc_bf16(void *out, const void *x, const void *w, const void *bias, const void *residual, int M, int N,
                   int K, cudaStream_t s);

// linear with an optional fused residual: out = round(res + round(x W^T + b)).
// `ref` selects the reference summation order (linear.cu).
int linear_forward(wginferDataType_t dtype, void *out, const void *x, const void *w, const void *bias,
                   const void *residual, int M, int N, int K, bool ref, cudaStream_t s);

// Batched decode attention over per-sequence KV caches (attention.cu). Row b
// of q [B, nh, dh] is the newest token of the sequence whose cache starts at
// kcache + b * seq_stride and holds lens[b] + 1 positions.
void attn_prepare();  // call outside graph capture, once per device
size_t attn_decode_workspace(int B, int nh, int nkvh, int dh, int maxlen, bool ref);
int attn_decode(wginferDataType_t dtype, void *out, const void *q, const void *kcache, const void *vcache,
                size_t seq_stride, const int64_t *lens, int B, int nh, int nkvh, int dh, int maxlen, float scale,
                void *ws, bool ref, cudaStream_t s, const void *pf_ptr = nullptr, size_t pf_bytes = 0);

// rope with a host-built {cos, sin} table [table_len][d/2] (rope.cu).
int rope_apply_table(wginferDataType_t dtype, void *out, const void *in, const int64_t *pos_ids, const float2 *table,
                     int table_len, int S, int H, int d, cudaStream_t s);

// Fused decode GEMV (decode_gemv.cu). Rows of x: M0 (processed 8 at a time).
struct DecodeGemvParams {
    const void *w;       // [N, K]
    const void *x;       // [M0, K]
    int M0, M, N, K;     // M is set per launch
    int groups;          // weight-row pairs this call covers
    // prologue RMS
    const void *norm_w;
    float eps;
    // epilogue STORE / SWIGLU
    void *out;           // [M0, ldo]
    int ldo;
    const void *bias;    // indexed by weight row, may be null
    const void *res;     // residual [M0, ldo] (STORE), may be null or alias out
    int di;              // SWIGLU: gate rows [0, di), up rows [di, 2 di)
    // epilogue ROPEKV
    const int64_t *pos;  // [M0]
    const float2 *table; // [maxseq][dh / 2]
    void *q_out;         // [M0, nh, dh]
    void *kc, *vc;       // cache of sequence 0 for this layer
    size_t seq_stride;   // elements per sequence in kc / vc
    int nh, nkvh, dh, maxseq, prefill_seq;
    unsigned long long *err;
    // weights of the kernels that follow, pulled into L2 while this one runs
    const void *pf_ptr[2];
    size_t pf_bytes[2];
    // [M0, K] scratch for the normalised rows when more than 8 rows take the
    // tensor-core path with the RMS prologue (may be null: GEMV chunks then)
    void *xn;
    // epilogue ARGMAX (the lm_head of a decode step): the logits are stored
    // as with STORE, and each CTA folds its rows' (value, index) keys into
    // amax_keys[m] (zero between launches); the CTA that finishes last writes
    // tokens[m] = argmax of row m, advances lens[m] (up to maxlen) and clears
    // the keys and amax_count
    unsigned long long *amax_keys;  // [M0]
    unsigned *amax_count;
    int64_t *tokens, *lens;
    int64_t maxlen;
};
enum { DG_PRO_PLAIN = 0, DG_PRO_RMS = 1, DG_EPI_STORE = 0, DG_EPI_SWIGLU = 1, DG_EPI_ROPEKV = 2, DG_EPI_ARGMAX = 3 };
int decode_gemv(wginferDataType_t dtype, const DecodeGemvParams &p, int pro, int epi, cudaStream_t s);
void decode_gemv_prepare();  // raises shared-memory limits; call outside graph capture

// The same projections and epilogues on the tensor cores, for bf16 with
// more than 8 rows (linear_tc.cu). Rows index x, out, pos, q_out and, when
// prefill_seq < 0, the sequence; the prologue must already be applied.
bool tc_gemm_ok(const DecodeGemvParams &p);
int tc_gemm(const DecodeGemvParams &p, int epi, cudaStream_t s);
void tc_gemm_prepare();

// REFERENCE-numerics decode kernels for up to kRefChainMaxM input rows
// (ref_decode.cu): the projections with every output one sequential f32
// chain over K (linear_cpu.cpp:86-99), weights streamed ahead of the chains
// into shared memory; prologue RMS and the STORE / SWIGLU / ROPEKV / ARGMAX
// epilogues as in DecodeGemvParams (bias starts the chain). ref_chain_ok:
// whether ref_chain_gemv takes these arguments (else use linear_forward).
constexpr int kRefChainMaxM = 4;
bool ref_chain_ok(wginferDataType_t dtype, const DecodeGemvParams &p);
int ref_chain_gemv(wginferDataType_t dtype, const DecodeGemvParams &p, int pro, int epi, cudaStream_t s);
// Decode attention over per-sequence caches in the reference's order
// (self_attention_cpu.cpp:37-89) for caches of up to ref_attn_max_len()
// positions; false from ref_attn_decode_ok: use attn_decode.
bool ref_attn_decode_ok(wginferDataType_t dtype, int nh, int nkvh, int dh, int maxlen, const void *kcache,
                        const void *vcache, size_t seq_stride);
int ref_attn_decode(wginferDataType_t dtype, void *out, const void *q, const void *kcache, const void *vcache,
                    size_t seq_stride, const int64_t *lens, int B, int nh, int nkvh, int dh, int maxlen, float scale,
                    cudaStream_t s);
void ref_decode_prepare();  // raises shared-memory limits; call outside graph capture

}  // namespace wgb
