// Test infrastructure only: a C-ABI veneer over the reference's own CPU code,
// compiled together with the reference sources into oracle/_ref/libwginfer_ref.so
// by oracle/Makefile. It is the checker the oracle restatement is pinned
// against, and the CPU baseline that bench.py times; nothing in the product
// links it.
//
// Every wrapper calls the reference function named in its comment unchanged.
#include "models/qwen2/model.hpp"
#include "ops/add/cpu/add_cpu.hpp"
#include "ops/argmax/cpu/argmax_cpu.hpp"
#include "ops/embedding/cpu/embedding_cpu.hpp"
#include "ops/linear/cpu/linear_cpu.hpp"
#include "ops/rms_norm/cpu/rms_norm_cpu.hpp"
#include "ops/rope/cpu/rope_cpu.hpp"
#include "ops/self_attention/cpu/self_attention_cpu.hpp"
#include "ops/swiglu/cpu/swiglu_cpu.hpp"

#include <cstring>
#include <exception>
#include <string>

using namespace wginfer;
namespace q2 = wginfer::models::qwen2;

#define REF_TRY(expr)                                                     \
    try {                                                                 \
        expr;                                                             \
        return 0;                                                         \
    } catch (const std::exception &e) {                                   \
        std::strncpy(g_err, e.what(), sizeof(g_err) - 1);                 \
        return 1;                                                         \
    }

static char g_err[512];

extern "C" {

const char *ref_last_error() { return g_err; }

// src/ops/add/cpu/add_cpu.cpp:19
int ref_add(void *c, const void *a, const void *b, int dtype, size_t numel) {
    REF_TRY(ops::cpu::add((std::byte *)c, (const std::byte *)a, (const std::byte *)b,
                          (wginferDataType_t)dtype, numel))
}

// src/ops/argmax/cpu/argmax_cpu.cpp:54
int ref_argmax(int64_t *max_idx, void *max_val, const void *vals, int dtype, size_t numel) {
    REF_TRY(ops::cpu::argmax(max_idx, (std::byte *)max_val, (const std::byte *)vals,
                             (wginferDataType_t)dtype, numel))
}

// src/ops/embedding/cpu/embedding_cpu.cpp:25
int ref_embedding(void *out, const int64_t *index, const void *weight, int dtype,
                  size_t index_numel, size_t embedding_dim) {
    REF_TRY(ops::cpu::embedding((std::byte *)out, (const std::byte *)index,
                                (const std::byte *)weight, (wginferDataType_t)dtype,
                                index_numel, embedding_dim))
}

// src/ops/linear/cpu/linear_cpu.cpp:180
int ref_linear(void *out, const void *in, const void *weight, const void *bias, int dtype,
               size_t M, size_t N, size_t K) {
    REF_TRY(ops::cpu::linear((std::byte *)out, (const std::byte *)in,
                             (const std::byte *)weight, (const std::byte *)bias,
                             (wginferDataType_t)dtype, M, N, K))
}

// src/ops/rms_norm/cpu/rms_norm_cpu.cpp:32
int ref_rms_norm(void *out, const void *in, const void *weight, int dtype, size_t M,
                 size_t N, float eps) {
    REF_TRY(ops::cpu::rms_norm((std::byte *)out, (const std::byte *)in,
                               (const std::byte *)weight, (wginferDataType_t)dtype, M, N,
                               eps))
}

// src/ops/rope/cpu/rope_cpu.cpp:43
int ref_rope(void *out, const void *in, const int64_t *pos_ids, int dtype, size_t seqlen,
             size_t nhead, size_t head_dim, float theta) {
    REF_TRY(ops::cpu::rope((std::byte *)out, (const std::byte *)in, pos_ids,
                           (wginferDataType_t)dtype, seqlen, nhead, head_dim, theta))
}

// src/ops/self_attention/cpu/self_attention_cpu.cpp:94
int ref_self_attention(void *attn_val, const void *q, const void *k, const void *v,
                       int dtype, size_t seqlen, size_t nhead, size_t nkvhead, size_t d,
                       size_t dv, size_t total_len, float scale) {
    REF_TRY(ops::cpu::self_attention((std::byte *)attn_val, (const std::byte *)q,
                                     (const std::byte *)k, (const std::byte *)v,
                                     (wginferDataType_t)dtype, seqlen, nhead, nkvhead, d,
                                     dv, total_len, scale))
}

// src/ops/swiglu/cpu/swiglu_cpu.cpp:17
int ref_swiglu(void *out, const void *gate, const void *up, int dtype, size_t numel) {
    REF_TRY(ops::cpu::swiglu((std::byte *)out, (const std::byte *)gate,
                             (const std::byte *)up, (wginferDataType_t)dtype, numel))
}

// ---- the reference Qwen2 model on the CPU device (src/models/qwen2/model.cpp) ----

struct RefMeta {
    int dtype;
    size_t nlayer, hs, nh, nkvh, dh, di, maxseq, voc;
    float epsilon, theta;
    int64_t end_token;
};

void *ref_qwen2_create(const RefMeta *m) {
    try {
        q2::ModelMeta meta{};
        meta.dtype = (wginferDataType_t)m->dtype;
        meta.nlayer = m->nlayer;
        meta.hs = m->hs;
        meta.nh = m->nh;
        meta.nkvh = m->nkvh;
        meta.dh = m->dh;
        meta.di = m->di;
        meta.maxseq = m->maxseq;
        meta.voc = m->voc;
        meta.epsilon = m->epsilon;
        meta.theta = m->theta;
        meta.end_token = m->end_token;
        return new q2::Model(meta, WGINFER_DEVICE_CPU, 0);
    } catch (const std::exception &e) {
        std::strncpy(g_err, e.what(), sizeof(g_err) - 1);
        return nullptr;
    }
}

void ref_qwen2_destroy(void *model) { delete (q2::Model *)model; }

// Loads one weight from host memory. `layer` < 0 selects a global weight
// (in_embed, out_embed, out_norm_w); names follow python/bindings/models/qwen2.cpp.
int ref_qwen2_set_weight(void *model, const char *name, int layer, const void *host,
                         const size_t *shape, int ndim) {
    try {
        auto *mdl = (q2::Model *)model;
        std::vector<size_t> shp(shape, shape + ndim);
        tensor_t t = Tensor::create(shp, mdl->meta().dtype, WGINFER_DEVICE_CPU, 0);
        t->load(host);
        auto &w = mdl->weights();
        std::string n(name);
        if (layer < 0) {
            if (n == "in_embed") w.in_embed = t;
            else if (n == "out_embed") w.out_embed = t;
            else if (n == "out_norm_w") w.out_norm_w = t;
            else throw std::invalid_argument("unknown global weight " + n);
            return 0;
        }
        size_t l = (size_t)layer;
        if (n == "attn_norm_w") w.attn_norm_w[l] = t;
        else if (n == "attn_q_w") w.attn_q_w[l] = t;
        else if (n == "attn_q_b") w.attn_q_b[l] = t;
        else if (n == "attn_k_w") w.attn_k_w[l] = t;
        else if (n == "attn_k_b") w.attn_k_b[l] = t;
        else if (n == "attn_v_w") w.attn_v_w[l] = t;
        else if (n == "attn_v_b") w.attn_v_b[l] = t;
        else if (n == "attn_o_w") w.attn_o_w[l] = t;
        else if (n == "mlp_norm_w") w.mlp_norm_w[l] = t;
        else if (n == "mlp_gate_w") w.mlp_gate_w[l] = t;
        else if (n == "mlp_up_w") w.mlp_up_w[l] = t;
        else if (n == "mlp_down_w") w.mlp_down_w[l] = t;
        else throw std::invalid_argument("unknown layer weight " + n);
        return 0;
    } catch (const std::exception &e) {
        std::strncpy(g_err, e.what(), sizeof(g_err) - 1);
        return 1;
    }
}

// src/models/qwen2/model.cpp:371 (Model::infer); greedy when top_k == 1.
int ref_qwen2_infer(void *model, const int64_t *token_ids, size_t ntoken, int64_t *next) {
    try {
        std::vector<int64_t> ids(token_ids, token_ids + ntoken);
        *next = ((q2::Model *)model)->infer(ids.data(), ids.size(), 1, 1.0f, 1.0f);
        return 0;
    } catch (const std::exception &e) {
        std::strncpy(g_err, e.what(), sizeof(g_err) - 1);
        return 1;
    }
}

void ref_qwen2_reset_cache(void *model) { ((q2::Model *)model)->reset_cache(); }

} // extern "C"
