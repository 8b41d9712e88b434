// tcgen05 tensor-core GEMM for linear (placeholder until the kernel lands).
#include "common.cuh"
#include "kernels.h"

namespace wgb {
bool linear_tc_supported(size_t, size_t, size_t, const void *, const void *, const void *) { return false; }
int linear_tc_bf16(void *, const void *, const void *, const void *, const void *, int, int, int, cudaStream_t) {
    return set_error(WGB_ERR_UNSUPPORTED, "tcgen05 linear not built");
}
}  // namespace wgb
