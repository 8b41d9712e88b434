// Status codes, per-thread error text, numerics mode and the device-side
// error record.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"

namespace wgb {

static thread_local char t_err[512] = "";
static thread_local int t_numerics = WGB_NUMERICS_FAST;

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(WGB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return WGB_OK;
}

int current_numerics() { return t_numerics; }

bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("WGB_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

int sm_count() {
    static thread_local int dev = -1, n = kNumSMs;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return kNumSMs;
    if (d != dev) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) == cudaSuccess && v > 0) n = v;
        dev = d;
    }
    return n;
}

// First recorded bad value: {code, value}. Code 1 = embedding index out of range.
__device__ unsigned long long g_dev_err[2];

unsigned long long *dev_error_ptr() {
    static thread_local int dev = -1;
    static thread_local unsigned long long *ptr = nullptr;
    int d = 0;
    cudaGetDevice(&d);
    if (d != dev) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_err) != cudaSuccess) return nullptr;
        ptr = (unsigned long long *)p;
        dev = d;
    }
    return ptr;
}

}  // namespace wgb

extern "C" {

const char *wgb_status_string(int s) {
    switch (s) {
    case WGB_OK: return "ok";
    case WGB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case WGB_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case WGB_ERR_CUDA: return "CUDA error";
    case WGB_ERR_OUT_OF_RANGE: return "out of range";
    case WGB_ERR_NO_MEMORY: return "out of memory";
    case WGB_ERR_TIMEOUT: return "timeout";
    case WGB_ERR_UNSUPPORTED: return "unsupported";
    default: return "unknown status";
    }
}

const char *wgb_last_error(void) { return wgb::t_err; }

int wgb_version(void) { return 1; }

int wgb_set_numerics(int mode) {
    if (mode != WGB_NUMERICS_FAST && mode != WGB_NUMERICS_REFERENCE)
        return wgb::set_error(WGB_ERR_INVALID_ARGUMENT, "numerics mode %d", mode);
    wgb::t_numerics = mode;
    return WGB_OK;
}

int wgb_get_numerics(void) { return wgb::t_numerics; }

int wgb_device_error(int64_t *code, int64_t *value, wginferStream_t stream) {
    WGB_REQUIRE(code != nullptr, WGB_ERR_INVALID_ARGUMENT, "wgb_device_error: null code");
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long h[2] = {0, 0};
    void *p = wgb::dev_error_ptr();
    if (p == nullptr) return wgb::check_launch("wgb_device_error");
    if (cudaMemcpyAsync(h, p, sizeof(h), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemsetAsync(p, 0, sizeof(h), s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return wgb::check_launch("wgb_device_error");
    *code = (int64_t)h[0];
    if (value) *value = (int64_t)h[1];
    return WGB_OK;
}

}  // extern "C"
