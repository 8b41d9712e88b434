// Row maps and output epilogues shared by the decode GEMV kernels
// (decode_gemv.cu: one launch per projection; decode_step.cu: the whole
// decode step in one persistent launch). See decode_gemv.cu for what each
// epilogue computes and the reference lines it reproduces.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace wgb {

enum Epi { EPI_STORE = DG_EPI_STORE, EPI_SWIGLU = DG_EPI_SWIGLU, EPI_ROPEKV = DG_EPI_ROPEKV, EPI_ARGMAX = DG_EPI_ARGMAX };

// Weight row pair g is rows (2g, 2g + 1) for every epilogue: the model stores
// q/k rows with rotation partners (j, j + dh/2) of a head next to each other
// and gate/up rows interleaved (qwen2.cu, set_weight), so a pair is always
// two adjacent rows and a block of pairs is one contiguous byte range.
template <int EPI>
__device__ __forceinline__ void row_map(const DecodeGemvParams &p, int g, int &r0, int &r1) {
    r0 = 2 * g;
    r1 = 2 * g + 1;
}

// Rows per row pair g of the fused q/k/v projection: g < P = (nh + nkvh) *
// dh/2 is the rotation pair (j, j + dh/2) of one q or k head, rotated with
// cs = {cos, sin}(pos, j) and written to q_rope or into the K cache; the
// other pairs are two consecutive v values for the V cache. pos and cs may be
// loaded early by the caller (they do not depend on the previous kernel).
template <typename T>
__device__ __forceinline__ void rope_kv_store(const DecodeGemvParams &p, int g, bool r1ok, int m, float s0, float s1,
                                              int64_t pos, float2 cs) {
    {
        if (pos < 0 || pos >= p.maxseq) {
            record_device_error(p.err, 3, pos);
            return;
        }
        const int seq = p.prefill_seq >= 0 ? p.prefill_seq : m;
        const int half = p.dh >> 1;
        const int P = (p.nh + p.nkvh) * half;
        T *kc = reinterpret_cast<T *>(p.kc) + (size_t)seq * p.seq_stride + (size_t)pos * p.nkvh * p.dh;
        T *vc = reinterpret_cast<T *>(p.vc) + (size_t)seq * p.seq_stride + (size_t)pos * p.nkvh * p.dh;
        const float a = Elem<T>::load(Elem<T>::store(s0));
        const float b = Elem<T>::load(Elem<T>::store(s1));
        if (g < P) {
            const int h = g / half, j = g - h * half;
            const float o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
            const float o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
            T *dst = h < p.nh ? reinterpret_cast<T *>(p.q_out) + ((size_t)m * p.nh + h) * p.dh
                              : kc + (size_t)(h - p.nh) * p.dh;
            stf(dst, j, o0);
            stf(dst, j + half, o1);
        } else {
            const int e = 2 * (g - P);
            stf(vc, e, a);
            if (r1ok) stf(vc, e + 1, b);
        }
    }
}

template <typename T, int EPI>
__device__ __forceinline__ void epilogue(const DecodeGemvParams &p, int g, int r0, int r1, bool r1ok, int m, float s0,
                                         float s1) {
    const T *bias = reinterpret_cast<const T *>(p.bias);
    if (bias) {
        s0 += ldf(bias, r0);
        if (r1ok) s1 += ldf(bias, r1);
    }
    if (EPI == EPI_STORE) {
        T *out = reinterpret_cast<T *>(p.out);
        const T *res = reinterpret_cast<const T *>(p.res);
        const size_t i0 = (size_t)m * p.ldo + r0, i1 = (size_t)m * p.ldo + r1;
        if (res) {
            s0 = __fadd_rn(ldf(res, i0), Elem<T>::load(Elem<T>::store(s0)));
            if (r1ok) s1 = __fadd_rn(ldf(res, i1), Elem<T>::load(Elem<T>::store(s1)));
        }
        stf(out, i0, s0);
        if (r1ok) stf(out, i1, s1);
    } else if (EPI == EPI_SWIGLU) {
        const float gg = Elem<T>::load(Elem<T>::store(s0));
        const float uu = Elem<T>::load(Elem<T>::store(s1));
        stf(reinterpret_cast<T *>(p.out), (size_t)m * p.ldo + g,
            __fdiv_rn(__fmul_rn(uu, gg), __fadd_rn(1.0f, expf(-gg))));
    } else if (EPI == EPI_ROPEKV) {
        const int64_t pos = p.pos[m];
        const int half = p.dh >> 1;
        const int P = (p.nh + p.nkvh) * half;
        float2 cs = make_float2(0.f, 0.f);
        if (g < P && pos >= 0 && pos < p.maxseq) cs = p.table[(size_t)pos * half + (g % half)];
        rope_kv_store<T>(p, g, r1ok, m, s0, s1, pos, cs);
    }
}

// Operands of the epilogue of a CTA's first row block, loaded early by the
// caller: the bias (before the wait for the previous kernel: it does not
// depend on it), the residual (right after the wait, so its round trip
// overlaps the dot products), and for RoPE the position and {cos, sin}.
struct EpiPre {
    float b0 = 0.f, b1 = 0.f;  // bias of rows r0, r1 (0 without bias)
    float q0 = 0.f, q1 = 0.f;  // residual at (m, r0), (m, r1) (STORE with residual)
    int64_t pos = 0;
    float2 cs = make_float2(0.f, 0.f);
};

template <typename T, int EPI>
__device__ __forceinline__ void epilogue_pre(const DecodeGemvParams &p, int g, int r0, int r1, bool r1ok, int m,
                                             float s0, float s1, const EpiPre &e) {
    if (p.bias) {
        s0 += e.b0;
        s1 += e.b1;
    }
    if (EPI == EPI_STORE) {
        T *out = reinterpret_cast<T *>(p.out);
        const size_t i0 = (size_t)m * p.ldo + r0, i1 = (size_t)m * p.ldo + r1;
        if (p.res) {
            s0 = __fadd_rn(e.q0, Elem<T>::load(Elem<T>::store(s0)));
            s1 = __fadd_rn(e.q1, Elem<T>::load(Elem<T>::store(s1)));
        }
        stf(out, i0, s0);
        if (r1ok) stf(out, i1, s1);
    } else if (EPI == EPI_SWIGLU) {
        const float gg = Elem<T>::load(Elem<T>::store(s0));
        const float uu = Elem<T>::load(Elem<T>::store(s1));
        stf(reinterpret_cast<T *>(p.out), (size_t)m * p.ldo + g,
            __fdiv_rn(__fmul_rn(uu, gg), __fadd_rn(1.0f, expf(-gg))));
    } else if (EPI == EPI_ROPEKV) {
        rope_kv_store<T>(p, g, r1ok, m, s0, s1, e.pos, e.cs);
    }
}

}  // namespace wgb
