/*
 * wgo.c — CPU oracle for the wGInfer decode path. TEST INFRASTRUCTURE ONLY
 * (see wgo.h). Each function restates the reference CPU code named in its
 * comment, keeping the reference's rounding points and summation order; the
 * loops are reorganised (row blocking, OpenMP over independent outputs) only
 * where that leaves every individual sum in the same order.
 */
#include "wgo.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

enum { DT_F16 = 12, DT_F32 = 13, DT_BF16 = 15 };

/* ---- scalar conversions: src/utils/types.cpp:6-83 ---- */

float wgo_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round to nearest even by adding 0x7FFF plus the kept LSB; NaN is not
 * special-cased, exactly as types.cpp:74-83. */
uint16_t wgo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static float f16_to_f32(uint16_t h) { /* types.cpp:6-38 */
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu;
    uint32_t u;
    if (e == 31) {
        u = sign | 0x7F800000u | (m << 13);
    } else if (e == 0) {
        if (m == 0) {
            u = sign;
        } else {
            e = -14;
            while ((m & 0x400u) == 0) {
                m <<= 1;
                e--;
            }
            m &= 0x3FFu;
            u = sign | ((uint32_t)(e + 127) << 23) | (m << 13);
        }
    } else {
        u = sign | ((uint32_t)(e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Truncating conversion (no rounding), types.cpp:40-64. */
static uint16_t f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    int32_t e = (int32_t)((u >> 23) & 0xFFu) - 127;
    uint32_t m = u & 0x7FFFFFu;
    if (e >= 16) {
        if (e == 128 && m != 0) return (uint16_t)(sign | 0x7E00u);
        return (uint16_t)(sign | 0x7C00u);
    } else if (e >= -14) {
        return (uint16_t)(sign | ((uint32_t)(e + 15) << 10) | (m >> 13));
    } else if (e >= -24) {
        m |= 0x800000u;
        m >>= (-14 - e);
        return (uint16_t)(sign | (m >> 13));
    }
    return sign;
}

static int dt_ok(int dt) { return dt == DT_F16 || dt == DT_F32 || dt == DT_BF16; }
static size_t dt_size(int dt) { return dt == DT_F32 ? 4 : 2; }

static inline float ld(const void *p, size_t i, int dt) {
    if (dt == DT_F32) return ((const float *)p)[i];
    if (dt == DT_BF16) return wgo_bf16_to_f32(((const uint16_t *)p)[i]);
    return f16_to_f32(((const uint16_t *)p)[i]);
}

static inline void st(void *p, size_t i, int dt, float v) {
    if (dt == DT_F32) ((float *)p)[i] = v;
    else if (dt == DT_BF16) ((uint16_t *)p)[i] = wgo_f32_to_bf16(v);
    else ((uint16_t *)p)[i] = f32_to_f16(v);
}

static void to_f32(float *dst, const void *src, size_t n, int dt) {
    for (size_t i = 0; i < n; i++) dst[i] = ld(src, i, dt);
}

/* ---- ops ---- */

/* src/ops/add/cpu/add_cpu.cpp:7-16: f32 add then one rounding. */
int wgo_add(void *c, const void *a, const void *b, int dt, size_t n) {
    if (!dt_ok(dt)) return 1;
#pragma omp parallel for schedule(static) if (n > (1u << 20))
    for (size_t i = 0; i < n; i++) st(c, i, dt, ld(a, i, dt) + ld(b, i, dt));
    return 0;
}

/* src/ops/argmax/cpu/argmax_cpu.cpp:13-51: first index of the maximum under
 * strict '>' (f16/bf16 compared as f32); empty input gives (0, 0). */
int wgo_argmax(int64_t *max_idx, void *max_val, const void *vals, int dt, size_t n) {
    if (!dt_ok(dt)) return 1;
    if (n == 0) {
        *max_idx = 0;
        st(max_val, 0, dt, 0.0f);
        return 0;
    }
    float best = ld(vals, 0, dt);
    size_t bi = 0;
    for (size_t i = 1; i < n; i++) {
        float v = ld(vals, i, dt);
        if (v > best) {
            best = v;
            bi = i;
        }
    }
    *max_idx = (int64_t)bi;
    memcpy(max_val, (const char *)vals + bi * dt_size(dt), dt_size(dt));
    return 0;
}

/* src/ops/embedding/cpu/embedding_cpu.cpp:10-22: row copy. The reference does
 * not check the index; the oracle rejects indices outside [0, vocab). */
int wgo_embedding(void *out, const int64_t *index, const void *weight, int dt, size_t ni,
                  size_t dim, size_t vocab) {
    if (!dt_ok(dt)) return 1;
    size_t rb = dim * dt_size(dt);
    for (size_t i = 0; i < ni; i++) {
        if (index[i] < 0 || (uint64_t)index[i] >= vocab) return 2;
        memcpy((char *)out + i * rb, (const char *)weight + (size_t)index[i] * rb, rb);
    }
    return 0;
}

/* src/ops/linear/cpu/linear_cpu.cpp:25-72 (f32, blocked) and :75-107 (f16/bf16,
 * naive). Both compute, for every output, s = 0 (+ bias), then
 * s = fl(s + fl(x[k] * w[k])) for k = 0..K-1 in order, then one rounding to
 * the output type. The blocked f32 loop stores and reloads s between
 * 64-wide k blocks, which does not change the order. */
int wgo_linear(void *out, const void *in, const void *w, const void *bias, int dt,
               size_t M, size_t N, size_t K) {
    if (!dt_ok(dt)) return 1;
    if (M == 0 || N == 0) return 0;
    float *xf = (float *)malloc(sizeof(float) * (M * K + 1));
    if (!xf) return 3;
    to_f32(xf, in, M * K, dt);
    if (M < 8) {
        /* four weight rows per step: four independent sequential chains */
#pragma omp parallel for schedule(static)
        for (size_t n0 = 0; n0 < N; n0 += 4) {
            size_t nn = (N - n0) < 4 ? (N - n0) : 4;
            for (size_t m = 0; m < M; m++) {
                float s[4] = {0.f, 0.f, 0.f, 0.f};
                for (size_t r = 0; r < nn; r++)
                    if (bias) s[r] += ld(bias, n0 + r, dt);
                const float *x = xf + m * K;
                if (nn == 4) {
                    for (size_t k = 0; k < K; k++) {
                        float xk = x[k];
                        s[0] += xk * ld(w, (n0 + 0) * K + k, dt);
                        s[1] += xk * ld(w, (n0 + 1) * K + k, dt);
                        s[2] += xk * ld(w, (n0 + 2) * K + k, dt);
                        s[3] += xk * ld(w, (n0 + 3) * K + k, dt);
                    }
                } else {
                    for (size_t r = 0; r < nn; r++)
                        for (size_t k = 0; k < K; k++) s[r] += x[k] * ld(w, (n0 + r) * K + k, dt);
                }
                for (size_t r = 0; r < nn; r++) st(out, m * N + n0 + r, dt, s[r]);
            }
        }
    } else {
        /* 16 input rows per chain bundle; x transposed so lanes are rows */
        size_t MB = (M + 15) / 16;
        float *xt = (float *)calloc(MB * K * 16, sizeof(float));
        if (!xt) {
            free(xf);
            return 3;
        }
        for (size_t m = 0; m < M; m++)
            for (size_t k = 0; k < K; k++) xt[((m / 16) * K + k) * 16 + (m % 16)] = xf[m * K + k];
#pragma omp parallel
        {
            float *wrow = (float *)malloc(sizeof(float) * (K + 1));
#pragma omp for schedule(static)
            for (size_t n = 0; n < N; n++) {
                to_f32(wrow, (const char *)w + n * K * dt_size(dt), K, dt);
                float b0 = bias ? ld(bias, n, dt) : 0.f;
                for (size_t mb = 0; mb < MB; mb++) {
                    float s[16];
                    for (int r = 0; r < 16; r++) s[r] = 0.f + b0;
                    const float *xb = xt + mb * K * 16;
                    for (size_t k = 0; k < K; k++) {
                        float wk = wrow[k];
                        for (int r = 0; r < 16; r++) s[r] += xb[k * 16 + r] * wk;
                    }
                    for (int r = 0; r < 16; r++) {
                        size_t m = mb * 16 + r;
                        if (m < M) st(out, m * N + n, dt, s[r]);
                    }
                }
            }
            free(wrow);
        }
        free(xt);
    }
    free(xf);
    return 0;
}

/* src/ops/rms_norm/cpu/rms_norm_cpu.cpp:9-29. */
int wgo_rms_norm(void *out, const void *in, const void *weight, int dt, size_t M, size_t N,
                 float eps) {
    if (!dt_ok(dt)) return 1;
#pragma omp parallel for schedule(static) if (M >= 64)
    for (size_t m = 0; m < M; m++) {
        float sum = 0.0f;
        for (size_t n = 0; n < N; n++) {
            float v = ld(in, m * N + n, dt);
            sum += v * v;
        }
        float mean = sum / (float)N;
        float scale = 1.0f / sqrtf(mean + eps);
        for (size_t n = 0; n < N; n++) {
            float v = ld(in, m * N + n, dt);
            float wv = ld(weight, n, dt);
            st(out, m * N + n, dt, v * wv * scale);
        }
    }
    return 0;
}

/* src/ops/rope/cpu/rope_cpu.cpp:8-40: half-split rotation of (j, j + d/2),
 * phi = pos / powf(theta, 2j/d). */
int wgo_rope(void *out, const void *in, const int64_t *pos_ids, int dt, size_t seqlen,
             size_t nhead, size_t d, float theta) {
    if (!dt_ok(dt) || (d & 1)) return 1;
    size_t half = d / 2;
    float *denom = (float *)malloc(sizeof(float) * (half + 1));
    for (size_t j = 0; j < half; j++) denom[j] = powf(theta, (2.0f * (float)j) / (float)d);
#pragma omp parallel for schedule(static) if (seqlen >= 64)
    for (size_t s = 0; s < seqlen; s++) {
        float p = (float)pos_ids[s];
        for (size_t h = 0; h < nhead; h++) {
            size_t off = (s * nhead + h) * d;
            for (size_t j = 0; j < half; j++) {
                float phi = p / denom[j];
                float sv = sinf(phi), cv = cosf(phi);
                float a = ld(in, off + j, dt), b = ld(in, off + j + half, dt);
                st(out, off + j, dt, a * cv - b * sv);
                st(out, off + j + half, dt, a * sv + b * cv);
            }
        }
    }
    free(denom);
    return 0;
}

/* src/ops/swiglu/cpu/swiglu_cpu.cpp:6-14: up * g / (1 + expf(-g)). */
int wgo_swiglu(void *out, const void *gate, const void *up, int dt, size_t n) {
    if (!dt_ok(dt)) return 1;
#pragma omp parallel for schedule(static) if (n > (1u << 20))
    for (size_t i = 0; i < n; i++) {
        float g = ld(gate, i, dt), u = ld(up, i, dt);
        st(out, i, dt, u * g / (1 + expf(-g)));
    }
    return 0;
}

/* src/ops/self_attention/cpu/self_attention_cpu.cpp:12-91. Per head: scores
 * scale * (sequential dot over d); keys j > i + (total_len - seqlen) get
 * -1e9; softmax with a sequential sum over every key; output = sequential sum
 * over keys of fl(p * v). Masked keys contribute exact zeros, so they are
 * skipped unless the whole row is masked (total_len < seqlen), where the
 * reference's uniform weights are reproduced literally. */
int wgo_self_attention(void *attn_val, const void *q, const void *k, const void *v, int dt,
                       size_t seqlen, size_t nhead, size_t nkvhead, size_t d, size_t dv,
                       size_t total_len, float scale) {
    if (!dt_ok(dt) || nkvhead == 0 || nhead % nkvhead) return 1;
    if (seqlen == 0 || total_len == 0) return 0;
    const long diag = (long)total_len - (long)seqlen;
#pragma omp parallel
    {
        float *sc = (float *)malloc(sizeof(float) * total_len);
        float *qf = (float *)malloc(sizeof(float) * d);
        float *acc = (float *)malloc(sizeof(float) * dv);
#pragma omp for schedule(dynamic) collapse(2)
        for (size_t h = 0; h < nhead; h++) {
            for (size_t i = 0; i < seqlen; i++) {
                const size_t kvh = h * nkvhead / nhead;
                for (size_t x = 0; x < d; x++) qf[x] = ld(q, (i * nhead + h) * d + x, dt);
                long last = (long)i + diag; /* last visible key */
                size_t nvis = last < 0 ? 0 : (size_t)(last + 1 < (long)total_len ? last + 1 : (long)total_len);
                size_t jend = nvis ? nvis : total_len;
                for (size_t j = 0; j < total_len; j++) {
                    if (j < nvis) {
                        float a = 0.f;
                        for (size_t x = 0; x < d; x++) a += qf[x] * ld(k, (j * nkvhead + kvh) * d + x, dt);
                        sc[j] = scale * a;
                    } else {
                        sc[j] = -1e9f;
                    }
                }
                float mx = sc[0];
                for (size_t j = 1; j < total_len; j++)
                    if (sc[j] > mx) mx = sc[j];
                float sum = 0.f;
                for (size_t j = 0; j < total_len; j++) {
                    sc[j] = expf(sc[j] - mx);
                    sum += sc[j];
                }
                for (size_t j = 0; j < total_len; j++) sc[j] /= sum;
                for (size_t m = 0; m < dv; m++) acc[m] = 0.f;
                for (size_t j = 0; j < jend; j++) {
                    float p = sc[j];
                    for (size_t m = 0; m < dv; m++) acc[m] += p * ld(v, (j * nkvhead + kvh) * dv + m, dt);
                }
                for (size_t m = 0; m < dv; m++) st(attn_val, (i * nhead + h) * dv + m, dt, acc[m]);
            }
        }
        free(sc);
        free(qf);
        free(acc);
    }
    return 0;
}

/* ---- Qwen2 model: src/models/qwen2/model.cpp:141-415 ---- */

typedef struct {
    wgo_meta m;
    wgo_weights w;
    const void **layer_ptrs; /* owned copy of the per-layer pointer tables */
    void **kc, **vc;          /* per-layer [maxseq, nkvh, dh] */
    size_t cache_len;
} wgo_model;

void *wgo_qwen2_create(const wgo_meta *meta, const wgo_weights *w) {
    if (!meta || !w || !dt_ok(meta->dtype) || meta->nkvh == 0 || meta->nh % meta->nkvh) return NULL;
    wgo_model *md = (wgo_model *)calloc(1, sizeof(wgo_model));
    md->m = *meta;
    md->w = *w;
    size_t L = meta->nlayer;
    md->layer_ptrs = (const void **)calloc(12 * L + 1, sizeof(void *));
    const void *const *src[12] = {w->attn_norm_w, w->attn_q_w, w->attn_q_b, w->attn_k_w,
                                  w->attn_k_b,    w->attn_v_w, w->attn_v_b, w->attn_o_w,
                                  w->mlp_norm_w,  w->mlp_gate_w, w->mlp_up_w, w->mlp_down_w};
    const void *const **dst[12] = {&md->w.attn_norm_w, &md->w.attn_q_w, &md->w.attn_q_b,
                                   &md->w.attn_k_w,    &md->w.attn_k_b, &md->w.attn_v_w,
                                   &md->w.attn_v_b,    &md->w.attn_o_w, &md->w.mlp_norm_w,
                                   &md->w.mlp_gate_w,  &md->w.mlp_up_w, &md->w.mlp_down_w};
    for (int t = 0; t < 12; t++) {
        for (size_t l = 0; l < L; l++) md->layer_ptrs[t * L + l] = src[t] ? src[t][l] : NULL;
        *dst[t] = md->layer_ptrs + t * L;
    }
    size_t es = dt_size(meta->dtype);
    md->kc = (void **)calloc(L, sizeof(void *));
    md->vc = (void **)calloc(L, sizeof(void *));
    for (size_t l = 0; l < L; l++) {
        md->kc[l] = calloc(meta->maxseq * meta->nkvh * meta->dh, es);
        md->vc[l] = calloc(meta->maxseq * meta->nkvh * meta->dh, es);
    }
    return md;
}

void wgo_qwen2_destroy(void *p) {
    wgo_model *md = (wgo_model *)p;
    if (!md) return;
    for (size_t l = 0; l < md->m.nlayer; l++) {
        free(md->kc[l]);
        free(md->vc[l]);
    }
    free(md->kc);
    free(md->vc);
    free(md->layer_ptrs);
    free(md);
}

void wgo_qwen2_reset_cache(void *p) { ((wgo_model *)p)->cache_len = 0; }

int wgo_qwen2_infer(void *p, const int64_t *ids, size_t S, float *last_logits, int64_t *next) {
    wgo_model *md = (wgo_model *)p;
    const wgo_meta *m = &md->m;
    const int dt = m->dtype;
    const size_t es = dt_size(dt), hs = m->hs, nh = m->nh, nkvh = m->nkvh, dh = m->dh, di = m->di;
    const size_t T = md->cache_len + S, old = md->cache_len;
    if (S == 0 || T > m->maxseq) return 1;
    int rc = 0;
    char *x = malloc(S * hs * es), *xn = malloc(S * hs * es), *tmp = malloc(S * hs * es);
    char *q = malloc(S * nh * dh * es), *qr = malloc(S * nh * dh * es);
    char *kf = malloc(S * nkvh * dh * es), *vf = malloc(S * nkvh * dh * es);
    char *att = malloc(S * nh * dh * es);
    char *g = malloc(S * di * es), *u = malloc(S * di * es);
    char *logits = malloc(m->voc * es);
    int64_t *pos = malloc(S * sizeof(int64_t));
    for (size_t i = 0; i < S; i++) pos[i] = (int64_t)(old + i);
    const float scale = 1.0f / sqrtf((float)dh);

    rc |= wgo_embedding(x, ids, md->w.in_embed, dt, S, hs, m->voc);
    for (size_t l = 0; l < m->nlayer && !rc; l++) {
        rc |= wgo_rms_norm(xn, x, md->w.attn_norm_w[l], dt, S, hs, m->epsilon);
        rc |= wgo_linear(q, xn, md->w.attn_q_w[l], md->w.attn_q_b[l], dt, S, nh * dh, hs);
        rc |= wgo_linear(kf, xn, md->w.attn_k_w[l], md->w.attn_k_b[l], dt, S, nkvh * dh, hs);
        rc |= wgo_linear(vf, xn, md->w.attn_v_w[l], md->w.attn_v_b[l], dt, S, nkvh * dh, hs);
        /* model.cpp:279-280: k then q; K is cached after RoPE, V as is */
        rc |= wgo_rope((char *)md->kc[l] + old * nkvh * dh * es, kf, pos, dt, S, nkvh, dh, m->theta);
        rc |= wgo_rope(qr, q, pos, dt, S, nh, dh, m->theta);
        memcpy((char *)md->vc[l] + old * nkvh * dh * es, vf, S * nkvh * dh * es);
        rc |= wgo_self_attention(att, qr, md->kc[l], md->vc[l], dt, S, nh, nkvh, dh, dh, T, scale);
        rc |= wgo_linear(tmp, att, md->w.attn_o_w[l], NULL, dt, S, hs, nh * dh);
        rc |= wgo_add(x, x, tmp, dt, S * hs);
        rc |= wgo_rms_norm(xn, x, md->w.mlp_norm_w[l], dt, S, hs, m->epsilon);
        rc |= wgo_linear(g, xn, md->w.mlp_gate_w[l], NULL, dt, S, di, hs);
        rc |= wgo_linear(u, xn, md->w.mlp_up_w[l], NULL, dt, S, di, hs);
        rc |= wgo_swiglu(g, g, u, dt, S * di);
        rc |= wgo_linear(tmp, g, md->w.mlp_down_w[l], NULL, dt, S, hs, di);
        rc |= wgo_add(x, x, tmp, dt, S * hs);
    }
    if (!rc) {
        /* model.cpp:360-365 computes logits for every row; rows are
         * independent, so only the last one is formed here. */
        rc |= wgo_rms_norm(xn, x + (S - 1) * hs * es, md->w.out_norm_w, dt, 1, hs, m->epsilon);
        rc |= wgo_linear(logits, xn, md->w.out_embed, NULL, dt, 1, m->voc, hs);
        char mv[4];
        rc |= wgo_argmax(next, mv, logits, dt, m->voc);
        if (last_logits)
            for (size_t i = 0; i < m->voc; i++) last_logits[i] = ld(logits, i, dt);
        if (!rc) md->cache_len = T;
    }
    free(x); free(xn); free(tmp); free(q); free(qr); free(kf); free(vf); free(att);
    free(g); free(u); free(logits); free(pos);
    return rc;
}
