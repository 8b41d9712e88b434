// rope: half-split rotary embedding (GPT-NeoX layout) of [seqlen, nhead, d].
//
// One thread owns the pair (j, j + d/2) of one position for every head, so
// the angle pos / theta^(2j/d) and its sine and cosine are formed once per
// (position, j) instead of once per element. The rotation is
// (a cos - b sin, a sin + b cos) with each product and sum rounded
// separately, as src/ops/rope/cpu/rope_cpu.cpp:27-37 does. FAST uses the
// f32 powf/sinf/cosf; REFERENCE evaluates them in double and rounds once.
// A table variant (rope_apply_table) serves the model, whose cos/sin table
// is built on the host with the reference's exact formula.
#include "common.cuh"
#include "kernels.h"

namespace wgb {
namespace {

template <typename T, bool kRef>
__global__ void __launch_bounds__(128) rope_kernel(T *out, const T *in, const int64_t *pos_ids, int seqlen,
                                                   int nhead, int d, float theta) {
    const int half = d >> 1;
    const int s = blockIdx.y;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < half; j += gridDim.x * blockDim.x) {
        const float p = (float)pos_ids[s];
        const float ex = __fdiv_rn(2.0f * (float)j, (float)d);
        float sv, cv;
        if (kRef) {
            const float den = pow_cr(theta, ex);
            const float phi = __fdiv_rn(p, den);
            sv = sin_cr(phi);
            cv = cos_cr(phi);
        } else {
            const float den = powf(theta, ex);
            const float phi = __fdiv_rn(p, den);
            sincosf(phi, &sv, &cv);
        }
        for (int h = 0; h < nhead; h++) {
            const size_t off = ((size_t)s * nhead + h) * d;
            const float a = ldf(in, off + j), b = ldf(in, off + j + half);
            stf(out, off + j, __fsub_rn(__fmul_rn(a, cv), __fmul_rn(b, sv)));
            stf(out, off + j + half, __fadd_rn(__fmul_rn(a, sv), __fmul_rn(b, cv)));
        }
    }
}

// table[pos][j] = {cos, sin} for j < d/2; rows of S positions x H heads.
template <typename T>
__global__ void __launch_bounds__(128) rope_table_kernel(T *out, const T *in, const int64_t *pos_ids,
                                                         const float2 *table, int table_len, int S, int H,
                                                         int d, unsigned long long *err) {
    const int half = d >> 1;
    const int s = blockIdx.y;
    int64_t p = pos_ids[s];
    if (p < 0 || p >= table_len) {
        if (threadIdx.x == 0 && blockIdx.x == 0) record_device_error(err, 2, p);
        p = 0;
    }
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < half * H; idx += gridDim.x * blockDim.x) {
        const int h = idx / half, j = idx - h * half;
        const float2 cs = table[(size_t)p * half + j];
        const size_t off = ((size_t)s * H + h) * d;
        const float a = ldf(in, off + j), b = ldf(in, off + j + half);
        stf(out, off + j, __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y)));
        stf(out, off + j + half, __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x)));
    }
}

}  // namespace

int rope_apply_table(wginferDataType_t dtype, void *out, const void *in, const int64_t *pos_ids, const float2 *table,
                     int table_len, int S, int H, int d, cudaStream_t s) {
    if (S == 0) return WGB_OK;
    dim3 grid((unsigned)(((d / 2) * H + 127) / 128), (unsigned)S);
    WGB_DISPATCH_FLOAT(dtype, T,
        rope_table_kernel<T><<<grid, 128, 0, s>>>((T *)out, (const T *)in, pos_ids, table, table_len, S, H, d,
                                                  dev_error_ptr()));
    return check_launch("rope_apply_table");
}

}  // namespace wgb

extern "C" int wgb_rope(void *out, const void *in, const int64_t *pos_ids, wginferDataType_t dtype, size_t seqlen,
                        size_t nhead, size_t head_dim, float theta, wginferStream_t stream) {
    if (seqlen == 0 || nhead == 0 || head_dim == 0) return WGB_OK;
    WGB_REQUIRE(out && in && pos_ids, WGB_ERR_INVALID_ARGUMENT, "wgb_rope: null pointer");
    WGB_REQUIRE(head_dim % 2 == 0, WGB_ERR_INVALID_ARGUMENT, "wgb_rope: head_dim must be even");
    WGB_REQUIRE(theta > 0.f, WGB_ERR_INVALID_ARGUMENT, "wgb_rope: theta must be positive");
    WGB_REQUIRE(seqlen < 65536u * 1024u && nhead < (1u << 20) && head_dim < (1u << 20), WGB_ERR_INVALID_ARGUMENT,
                "wgb_rope: size too large");
    const int half = (int)head_dim / 2;
    dim3 grid((unsigned)((half + 127) / 128), (unsigned)seqlen);
    if (seqlen > 65535) return wgb::set_error(WGB_ERR_INVALID_ARGUMENT, "wgb_rope: seqlen > 65535");
    cudaStream_t s = (cudaStream_t)stream;
    const bool ref = wgb::current_numerics() == WGB_NUMERICS_REFERENCE;
    WGB_DISPATCH_FLOAT(dtype, T,
        if (ref) wgb::rope_kernel<T, true><<<grid, 128, 0, s>>>((T *)out, (const T *)in, pos_ids, (int)seqlen,
                                                                (int)nhead, (int)head_dim, theta);
        else wgb::rope_kernel<T, false><<<grid, 128, 0, s>>>((T *)out, (const T *)in, pos_ids, (int)seqlen,
                                                             (int)nhead, (int)head_dim, theta));
    return wgb::check_launch("wgb_rope");
}
