// embedding: out[i, :] = weight[index[i], :], a bit copy of whole rows.
//
// A warp copies one row with 16-byte loads/stores (any element type, since
// it moves bytes); rows whose byte length or addresses are not 16-byte
// multiples use 4- or 2-byte words. An index outside [0, vocab) zero-fills
// its row and is recorded in the device error word (the reference reads out
// of bounds there, src/ops/embedding/nvidia/embedding_nvidia.cu:10-24).
// Roofline: HBM, 2*T*dim*size + 8*T bytes.
#include "common.cuh"

namespace wgb {
namespace {

template <typename W>
__global__ void __launch_bounds__(256) embedding_kernel(char *out, const int64_t *index, const char *weight,
                                                        size_t nrows, size_t row_words, size_t vocab,
                                                        unsigned long long *err) {
    const size_t warp = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
    for (size_t i = warp; i < nrows; i += nwarps) {
        const int64_t id = index[i];
        W *dst = reinterpret_cast<W *>(out) + i * row_words;
        if (id < 0 || (uint64_t)id >= vocab) {
            if (lane == 0) record_device_error(err, 1, id);
            W z;
            memset(&z, 0, sizeof(W));
            for (size_t k = lane; k < row_words; k += 32) dst[k] = z;
            continue;
        }
        const W *src = reinterpret_cast<const W *>(weight) + (size_t)id * row_words;
        // up to 8 words per lane are requested before the first store (a
        // store may alias a later load, so a load-store loop would wait
        // for every word in turn)
        constexpr int kU = 8;
        for (size_t k0 = lane; k0 < row_words; k0 += 32 * kU) {
            W r[kU];
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (k0 + 32 * u < row_words) r[u] = src[k0 + 32 * u];
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (k0 + 32 * u < row_words) dst[k0 + 32 * u] = r[u];
        }
    }
}

}  // namespace
}  // namespace wgb

extern "C" int wgb_embedding(void *out, const int64_t *index, const void *weight, wginferDataType_t dtype,
                             size_t index_numel, size_t embedding_dim, size_t vocab, wginferStream_t stream) {
    if (index_numel == 0 || embedding_dim == 0) return WGB_OK;
    WGB_REQUIRE(out && index && weight, WGB_ERR_INVALID_ARGUMENT, "wgb_embedding: null pointer");
    size_t es;
    switch (dtype) {
    case WGINFER_DTYPE_F32: es = 4; break;
    case WGINFER_DTYPE_BF16:
    case WGINFER_DTYPE_F16: es = 2; break;
    default: return wgb::set_error(WGB_ERR_UNSUPPORTED_DTYPE, "wgb_embedding: dtype %d", (int)dtype);
    }
    const size_t row_bytes = embedding_dim * es;
    const uintptr_t al = (uintptr_t)out | (uintptr_t)weight | (uintptr_t)row_bytes;
    const size_t want = (index_numel + 7) / 8;
    const int cap = wgb::sm_count() * 8;
    const int blocks = (int)(want < (size_t)cap ? want : cap);
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long *err = wgb::dev_error_ptr();
    if ((al & 15) == 0)
        wgb::embedding_kernel<uint4><<<blocks, 256, 0, s>>>((char *)out, index, (const char *)weight, index_numel,
                                                            row_bytes / 16, vocab, err);
    else if ((al & 3) == 0)
        wgb::embedding_kernel<uint32_t><<<blocks, 256, 0, s>>>((char *)out, index, (const char *)weight, index_numel,
                                                               row_bytes / 4, vocab, err);
    else
        wgb::embedding_kernel<uint16_t><<<blocks, 256, 0, s>>>((char *)out, index, (const char *)weight, index_numel,
                                                               row_bytes / 2, vocab, err);
    return wgb::check_launch("wgb_embedding");
}
