// Internal entry points shared between translation units (not exported).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "wginfer_b200.h"

namespace wgb {

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
                void *ws, bool ref, cudaStream_t s);

// rope with a host-built {cos, sin} table [table_len][d/2] (rope.cu).
int rope_apply_table(wginferDataType_t dtype, void *out, const void *in, const int64_t *pos_ids, const float2 *table,
                     int table_len, int S, int H, int d, cudaStream_t s);

}  // namespace wgb
