/*
 * wginfer_b200.h — C-ABI of the B200 (sm_100a) device backend for the wGInfer
 * decode path.
 *
 * Each op entry point replaces the reference's NVIDIA backend function named
 * beside it (paths relative to the wGInfer tree); the reference's op front
 * (src/ops/<op>/op.cpp) keeps its validation and calls these with the same
 * raw device pointers, dtype and sizes. Differences from the reference
 * signatures: every call takes the stream to launch on (the reference always
 * used the legacy default stream) and returns a status instead of throwing.
 *
 * Conventions
 *  - Pointers are device pointers unless a parameter says "host".
 *  - dtype is F32, BF16 or F16 for floating tensors; indices are int64.
 *  - Return value: WGB_OK (0) or a wgbStatus_t; the message of the last
 *    failure on the calling thread is available from wgb_last_error().
 *  - Calls are asynchronous with respect to the host and never allocate
 *    device memory unless the comment says so.
 *  - Numerics: WGB_NUMERICS_FAST (default) accumulates in f32 in whatever
 *    order is fastest; WGB_NUMERICS_REFERENCE reproduces the reference CPU
 *    backend's sequential f32 summation order and rounding points, so bf16
 *    results are bit-identical to it (see wgb_set_numerics).
 */
#ifndef WGINFER_B200_H
#define WGINFER_B200_H

#include "wginfer.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    WGB_OK = 0,
    WGB_ERR_INVALID_ARGUMENT = 1,
    WGB_ERR_UNSUPPORTED_DTYPE = 2,
    WGB_ERR_CUDA = 3,
    WGB_ERR_OUT_OF_RANGE = 4,
    WGB_ERR_NO_MEMORY = 5,
    WGB_ERR_TIMEOUT = 6,
    WGB_ERR_UNSUPPORTED = 7,
} wgbStatus_t;

typedef enum {
    WGB_NUMERICS_FAST = 0,
    WGB_NUMERICS_REFERENCE = 1,
} wgbNumerics_t;

__export const char *wgb_status_string(int status);
/* Message of the most recent failure on the calling host thread. */
__export const char *wgb_last_error(void);
__export int wgb_version(void);

/* Per host thread, like cublasSetMathMode. REFERENCE mode: linear, rms_norm
 * and self_attention sum in the reference CPU order (src/ops/linear/cpu/
 * linear_cpu.cpp:75-107, rms_norm_cpu.cpp:9-29, self_attention_cpu.cpp:12-91);
 * exp/sin/cos/pow are evaluated in double precision and rounded once. */
__export int wgb_set_numerics(int mode);
__export int wgb_get_numerics(void);

/* Device-side error record: kernels that find bad data (an embedding index
 * outside [0, vocab)) record the first offending value here instead of
 * faulting. Reads and clears it; *code is 0 when nothing was recorded.
 * Codes: 1 embedding index out of range (value = the index); 2 rope
 * position outside its table; 3 decode position outside the KV cache
 * (value = the position); 6 a tensor-core
 * linear tile whose copy pipeline stalled (value = the tile's block index).
 * Synchronises `stream`. */
__export int wgb_device_error(int64_t *code, int64_t *value, wginferStream_t stream);

/* ---- ops ---------------------------------------------------------------- */

/* c = a + b elementwise. Replaces ops::nvidia::add (src/ops/add/nvidia/add_nvidia.cuh:11). */
__export int wgb_add(void *c, const void *a, const void *b, wginferDataType_t dtype, size_t numel,
                     wginferStream_t stream);

/* (first index of the maximum, maximum) of a 1-D vector; empty input gives
 * (0, 0). Replaces ops::nvidia::argmax (src/ops/argmax/nvidia/argmax_nvidia.cuh:10-14). */
__export int wgb_argmax(int64_t *max_idx, void *max_val, const void *vals,
                        wginferDataType_t dtype, size_t numel, wginferStream_t stream);

/* Row-wise argmax over vals[rows, numel] (contiguous): max_idx[rows],
 * max_val[rows] (max_val may be NULL). New entry for batched decode; each row
 * has the semantics of wgb_argmax. */
__export int wgb_argmax_rows(int64_t *max_idx, void *max_val, const void *vals,
                             wginferDataType_t dtype, size_t rows, size_t numel,
                             wginferStream_t stream);

/* Row-wise sampling over logits[rows, vocab] (contiguous) into out_idx[rows]
 * with the rules of the reference's host sampler sample_from_logits
 * (src/models/qwen2/model.cpp:60-137), which copies the logits to the host
 * and sorts them; here the whole draw stays on the device. temperature <= 0,
 * or top_k == 1 with top_p >= 1, gives the argmax; top_k outside [1, vocab]
 * means vocab; top_p outside (0, 1] means 1. Logits that compare equal are
 * ordered by index; NaN logits are never drawn unless all are NaN. The
 * random number of row r is a hash of (seed, offset, r): the same arguments
 * give the same tokens. New entry for batched decode. */
__export int wgb_sample_rows(int64_t *out_idx, const void *logits, wginferDataType_t dtype, size_t rows,
                             size_t vocab, int top_k, float top_p, float temperature, unsigned long long seed,
                             unsigned long long offset, wginferStream_t stream);

/* out[i, :] = weight[index[i], :]. Replaces ops::nvidia::embedding
 * (src/ops/embedding/nvidia/embedding_nvidia.cuh:6-8); `vocab` (weight rows,
 * known to the op front as weight->shape()[0]) is added so that an index
 * outside [0, vocab) zero-fills its row and is recorded for
 * wgb_device_error instead of reading out of bounds. */
__export int wgb_embedding(void *out, const int64_t *index, const void *weight,
                           wginferDataType_t dtype, size_t index_numel, size_t embedding_dim,
                           size_t vocab, wginferStream_t stream);

/* out[M, N] = in[M, K] . weight[N, K]^T (+ bias[N]), f32 accumulation, one
 * rounding of (sum + bias). bias may be NULL. Replaces ops::nvidia::linear
 * (src/ops/linear/nvidia/linear_nvidia.cuh:6-8). */
__export int wgb_linear(void *out, const void *in, const void *weight, const void *bias,
                        wginferDataType_t dtype, size_t M, size_t N, size_t K,
                        wginferStream_t stream);

/* out = in * weight * (mean(in^2) + eps)^-1/2 per row of in[M, N].
 * Replaces ops::nvidia::rms_norm (src/ops/rms_norm/nvidia/rms_norm_nvidia.cuh:5-6). */
__export int wgb_rms_norm(void *out, const void *in, const void *weight, wginferDataType_t dtype,
                          size_t M, size_t N, float eps, wginferStream_t stream);

/* Half-split rotary embedding of in[seqlen, nhead, head_dim] at positions
 * pos_ids[seqlen] (int64), angle pos / theta^(2j/head_dim). in may equal out.
 * Replaces ops::nvidia::rope (src/ops/rope/nvidia/rope_nvidia.cuh:8-10). */
__export int wgb_rope(void *out, const void *in, const int64_t *pos_ids, wginferDataType_t dtype,
                      size_t seqlen, size_t nhead, size_t head_dim, float theta,
                      wginferStream_t stream);

/* Causal GQA attention: q[seqlen, nhead, d], k[total_len, nkvhead, d],
 * v[total_len, nkvhead, dv] -> attn_val[seqlen, nhead, dv]; query i sees
 * keys j <= i + total_len - seqlen; head h reads kv head h*nkvhead/nhead.
 * Replaces ops::nvidia::self_attention
 * (src/ops/self_attention/nvidia/self_attention_nvidia.cuh:7-19).
 * Uses a library-owned device workspace that is allocated on first use and
 * grown when needed; callers that must not allocate use
 * wgb_self_attention_ex. */
__export int wgb_self_attention(void *attn_val, const void *q, const void *k, const void *v,
                                wginferDataType_t dtype, size_t seqlen, size_t nhead,
                                size_t nkvhead, size_t d, size_t dv, size_t total_len,
                                float scale, wginferStream_t stream);

/* Bytes of workspace wgb_self_attention_ex needs for these sizes (0 allowed). */
__export size_t wgb_self_attention_workspace_size(size_t seqlen, size_t nhead, size_t nkvhead,
                                                  size_t d, size_t dv, size_t total_len);

/* wgb_self_attention with caller-provided workspace (16-byte aligned, at
 * least wgb_self_attention_workspace_size bytes). Allocates nothing. */
__export int wgb_self_attention_ex(void *attn_val, const void *q, const void *k, const void *v,
                                   wginferDataType_t dtype, size_t seqlen, size_t nhead,
                                   size_t nkvhead, size_t d, size_t dv, size_t total_len,
                                   float scale, void *workspace, size_t workspace_bytes,
                                   wginferStream_t stream);

/* wgb_self_attention for callers that cannot allocate device memory: code
 * running inside an allocator or memory-pool callback (allocating there would
 * re-enter the allocator), host runtimes that own all device memory and give
 * their kernels no allocation hook, and threads that must not block in the
 * driver. No counterpart in the reference. Its scratch is one file-scope
 * device array of wgb_self_attention_noalloc_max_scratch() bytes (4 MiB),
 * held by every GPU that loads the library until exit; sizes whose scratch
 * would exceed it return WGB_ERR_OUT_OF_RANGE. Every call looks up the
 * array's device address (cudaGetSymbolAddress) with the caller's device
 * current; the first call on a device also loads the library's device code
 * there, so make that first call before any stream capture. Calls allocate
 * nothing. The scratch holds REFERENCE numerics' one score per key for caches
 * longer than shared memory holds. All calls on a device share the array,
 * which keeps the last call's contents; nothing in it has to start at zero
 * (every score a call reads is written earlier in that call), but calls whose
 * kernels overlap on the same device, e.g. on two streams, race: serialise
 * them, e.g. on one stream. */
__export int wgb_self_attention_noalloc(void *attn_val, const void *q, const void *k, const void *v,
                                        wginferDataType_t dtype, size_t seqlen, size_t nhead,
                                        size_t nkvhead, size_t d, size_t dv, size_t total_len,
                                        float scale, wginferStream_t stream);
__export size_t wgb_self_attention_noalloc_max_scratch(void);

/* out = up * gate / (1 + exp(-gate)). Replaces ops::nvidia::swiglu
 * (src/ops/swiglu/nvidia/swiglu_nvidia.cuh:6-7). */
__export int wgb_swiglu(void *out, const void *gate, const void *up, wginferDataType_t dtype,
                        size_t numel, wginferStream_t stream);

/* ---- Qwen2 decoder (the caller of the ops; src/models/qwen2/model.hpp) ---- */

typedef struct {
    int dtype; /* wginferDataType_t; BF16 or F32 */
    size_t nlayer, hs, nh, nkvh, dh, di, maxseq, voc;
    float epsilon, theta;
    int64_t end_token;
} wgbQwen2Meta;

typedef struct wgbQwen2Model wgbQwen2Model;

/* Creates a model on `device` holding `max_batch` independent sequences, each
 * with a KV cache of meta->maxseq positions. Allocates one device arena for
 * weights, caches and activations. */
__export int wgb_qwen2_create(const wgbQwen2Meta *meta, int device, int max_batch,
                              wgbQwen2Model **model);
__export int wgb_qwen2_destroy(wgbQwen2Model *model);

/* Copies one weight in. Names and shapes are those of the reference's
 * ModelWeights (model.hpp:34-60): global "in_embed", "out_embed",
 * "out_norm_w" (layer = -1) and per layer "attn_norm_w", "attn_q_w",
 * "attn_q_b", "attn_k_w", "attn_k_b", "attn_v_w", "attn_v_b", "attn_o_w",
 * "mlp_norm_w", "mlp_gate_w", "mlp_up_w", "mlp_down_w". `src` is host memory
 * when src_on_host, else device memory; `bytes` must equal the weight size. */
__export int wgb_qwen2_set_weight(wgbQwen2Model *model, const char *name, int layer,
                                  const void *src, size_t bytes, int src_on_host);

/* Forgets the KV cache of every sequence (model.cpp:328-330). */
__export int wgb_qwen2_reset_cache(wgbQwen2Model *model);

/* Model::infer for sequence 0 (model.cpp:371-415): token_ids are host
 * memory; runs them through the model (prefill when ntoken > 1), appends to
 * the KV cache and returns the next token in *next (host). Greedy when
 * top_k == 1, top_p >= 1 and temperature == 1, else samples from the last
 * row's logits on the device with the reference's rules (wgb_sample_rows);
 * only the drawn token is copied back. Synchronises the model stream. */
__export int wgb_qwen2_infer(wgbQwen2Model *model, const int64_t *token_ids, size_t ntoken,
                             int top_k, float top_p, float temperature, int64_t *next);

/* Device-resident decode for sequences [0, batch): reads each sequence's
 * current token from the model's device token buffer, runs one decode step
 * for all of them and writes the greedy next tokens back to that buffer, all
 * on the model stream without host synchronisation. The step is captured
 * once per batch size into a CUDA graph and replayed. */
__export int wgb_qwen2_decode_step(wgbQwen2Model *model, int batch);

/* Prefill of sequence `seq` with host token_ids; leaves the greedy next token
 * in the device token buffer slot `seq`. */
__export int wgb_qwen2_prefill(wgbQwen2Model *model, int seq, const int64_t *token_ids,
                               size_t ntoken);

/* Device token buffer (int64[max_batch]) and the model stream, for callers
 * that stage tokens themselves. */
__export int64_t *wgb_qwen2_token_buffer(wgbQwen2Model *model);
__export wginferStream_t wgb_qwen2_stream(wgbQwen2Model *model);
/* Current KV length of sequence `seq`. */
__export size_t wgb_qwen2_cache_len(wgbQwen2Model *model, int seq);
/* Device pointer to the last logits row of sequence `seq` (dtype, voc). */
__export const void *wgb_qwen2_logits(wgbQwen2Model *model, int seq);
/* One decode step (like wgb_qwen2_decode_step) launched eagerly with a CUDA
 * event after every launch, for a per-launch device-time breakdown: us[i]
 * is the time of launch i (microseconds) and names holds one launch name per
 * line. Events between launches serialise them, so the sum exceeds a graph
 * step; the shares are what it is for. */
__export int wgb_qwen2_trace_step(wgbQwen2Model *model, int batch, int max_launches, float *us, char *names,
                                  size_t names_cap, int *n_launches);

/* Synchronous host copies of the token buffer (int64[batch]) and of the
 * last logits row of `seq` widened to f32 (voc floats). */
__export int wgb_qwen2_read_tokens(wgbQwen2Model *model, int64_t *host, int batch);
__export int wgb_qwen2_read_logits(wgbQwen2Model *model, int seq, float *host);

#ifdef __cplusplus
}
#endif
#endif /* WGINFER_B200_H */
