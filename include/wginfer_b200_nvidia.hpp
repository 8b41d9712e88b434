// wginfer_b200_nvidia.hpp — drop-in C++ shim for the reference's NVIDIA op
// backend.
//
// Defines wginfer::ops::nvidia::<op> with exactly the signatures of the
// reference's headers (src/ops/<op>/nvidia/<op>_nvidia.cuh), forwarding to
// the C-ABI in wginfer_b200.h. A maintainer includes this header instead of
// the reference's .cuh files and links libwginfer_b200.so; src/ops/*/op.cpp
// and the Qwen2 model compile unchanged. Errors are rethrown with the
// reference's exception types (std::invalid_argument for bad arguments,
// std::runtime_error otherwise). `stream()` picks the stream to launch on;
// the reference launched on the legacy default stream, which is the default
// here too.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "wginfer_b200.h"

namespace wginfer::ops::nvidia {

inline wginferStream_t &stream() {
    static thread_local wginferStream_t s = nullptr;
    return s;
}

inline void wgb_check(int status, const char *op) {
    if (status == WGB_OK) return;
    std::string msg = std::string(op) + ": " + wgb_last_error();
    if (status == WGB_ERR_INVALID_ARGUMENT || status == WGB_ERR_OUT_OF_RANGE) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

inline void add(std::byte *c, const std::byte *a, const std::byte *b, wginferDataType_t type, size_t numel) {
    wgb_check(wgb_add(c, a, b, type, numel, stream()), "add");
}

inline void argmax(int64_t *max_idx, std::byte *max_val, const std::byte *vals, wginferDataType_t type,
                   size_t numel) {
    wgb_check(wgb_argmax(max_idx, max_val, vals, type, numel, stream()), "argmax");
}

// The reference signature has no vocabulary size; without it the row bound
// cannot be checked, so pass SIZE_MAX (the op front knows weight->shape()[0]
// and should call the overload below).
inline void embedding(std::byte *out, const std::byte *index, const std::byte *weight, wginferDataType_t type,
                      size_t index_numel, size_t embedding_dim, size_t vocab = SIZE_MAX) {
    wgb_check(wgb_embedding(out, reinterpret_cast<const int64_t *>(index), weight, type, index_numel, embedding_dim,
                            vocab, stream()),
              "embedding");
}

inline void linear(std::byte *out, const std::byte *in, const std::byte *weight, const std::byte *bias,
                   wginferDataType_t type, size_t M, size_t N, size_t K) {
    wgb_check(wgb_linear(out, in, weight, bias, type, M, N, K, stream()), "linear");
}

inline void rms_norm(std::byte *out, const std::byte *in, const std::byte *weight, wginferDataType_t type, size_t M,
                     size_t N, float eps) {
    wgb_check(wgb_rms_norm(out, in, weight, type, M, N, eps, stream()), "rms_norm");
}

inline void rope(std::byte *out, const std::byte *in, const int64_t *pos_ids, wginferDataType_t type, size_t seqlen,
                 size_t nhead, size_t head_dim, float theta) {
    wgb_check(wgb_rope(out, in, pos_ids, type, seqlen, nhead, head_dim, theta, stream()), "rope");
}

inline void self_attention(std::byte *attn_val, const std::byte *q, const std::byte *k, const std::byte *v,
                           wginferDataType_t type, size_t seqlen, size_t nhead, size_t nkvhead, size_t d, size_t dv,
                           size_t total_len, float scale) {
    wgb_check(wgb_self_attention(attn_val, q, k, v, type, seqlen, nhead, nkvhead, d, dv, total_len, scale, stream()),
              "self_attention");
}

inline void swiglu(std::byte *out, const std::byte *gate, const std::byte *up, wginferDataType_t type, size_t numel) {
    wgb_check(wgb_swiglu(out, gate, up, type, numel, stream()), "swiglu");
}

}  // namespace wginfer::ops::nvidia
