/*
 * wgo — CPU oracle for the wGInfer decode path. TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU backend (src/ops/<op>/cpu and
 * src/models/qwen2/model.cpp) with the same arithmetic in the same order:
 * f32 accumulation, one rounding per reference rounding, sequential sums in
 * the reference's index order, the reference's bf16 (round-to-nearest-even,
 * no NaN case) and f16 (truncating) conversions, and the C library's
 * expf/powf/sinf/cosf. It is pinned against the reference's own code built
 * from source (oracle/_ref) and against committed golden fixtures.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker. The product never calls it.
 *
 * dtype codes are wginferDataType_t values: F16 = 12, F32 = 13, BF16 = 15.
 * Every function returns 0 on success and nonzero on a bad argument.
 */
#ifndef WGO_H
#define WGO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int wgo_add(void *c, const void *a, const void *b, int dtype, size_t numel);
int wgo_argmax(int64_t *max_idx, void *max_val, const void *vals, int dtype, size_t numel);
int wgo_embedding(void *out, const int64_t *index, const void *weight, int dtype,
                  size_t index_numel, size_t embedding_dim, size_t vocab);
int wgo_linear(void *out, const void *in, const void *weight, const void *bias, int dtype,
               size_t M, size_t N, size_t K);
int wgo_rms_norm(void *out, const void *in, const void *weight, int dtype, size_t M,
                 size_t N, float eps);
int wgo_rope(void *out, const void *in, const int64_t *pos_ids, int dtype, size_t seqlen,
             size_t nhead, size_t head_dim, float theta);
int wgo_self_attention(void *attn_val, const void *q, const void *k, const void *v,
                       int dtype, size_t seqlen, size_t nhead, size_t nkvhead, size_t d,
                       size_t dv, size_t total_len, float scale);
int wgo_swiglu(void *out, const void *gate, const void *up, int dtype, size_t numel);

/* Qwen2 decoder (src/models/qwen2/model.{hpp,cpp}). Weight pointers are host
 * arrays of `dtype` and stay owned by the caller for the model's lifetime.
 * Optional biases may be NULL. */
typedef struct {
    int dtype;
    size_t nlayer, hs, nh, nkvh, dh, di, maxseq, voc;
    float epsilon, theta;
    int64_t end_token;
} wgo_meta;

typedef struct {
    const void *in_embed, *out_embed, *out_norm_w;
    const void *const *attn_norm_w, *const *attn_q_w, *const *attn_q_b;
    const void *const *attn_k_w, *const *attn_k_b, *const *attn_v_w, *const *attn_v_b;
    const void *const *attn_o_w, *const *mlp_norm_w, *const *mlp_gate_w;
    const void *const *mlp_up_w, *const *mlp_down_w;
} wgo_weights;

void *wgo_qwen2_create(const wgo_meta *meta, const wgo_weights *w);
void wgo_qwen2_destroy(void *model);
void wgo_qwen2_reset_cache(void *model);
/* Runs `ntoken` tokens through the model (prefill when > 1), appends their
 * K/V to the cache, writes the last row's logits (f32, voc entries, may be
 * NULL) and the greedy next token. */
int wgo_qwen2_infer(void *model, const int64_t *token_ids, size_t ntoken,
                    float *last_logits, int64_t *next_token);

/* bf16 helpers used by the tests. */
uint16_t wgo_f32_to_bf16(float f);
float wgo_bf16_to_f32(uint16_t h);

#ifdef __cplusplus
}
#endif
#endif
