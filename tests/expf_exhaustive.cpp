// Checks wgb::expf_glibc (wginfer_b200/csrc/libm_expf.cuh, compiled here as
// host code) against the host C library's expf on every 32-bit pattern, or on
// every `stride`-th one. Prints the number of differing results (NaN results
// compare equal to any NaN) and the first few inputs that differ.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "libm_expf.cuh"

int main(int argc, char **argv) {
    const unsigned long long stride = argc > 1 ? strtoull(argv[1], nullptr, 10) : 1;
    unsigned long long bad = 0, checked = 0;
#pragma omp parallel for reduction(+ : bad, checked) schedule(static)
    for (long long i = 0; i < (1LL << 32); i += (long long)stride) {
        const uint32_t u = (uint32_t)i;
        float x;
        memcpy(&x, &u, 4);
        const float want = expf(x), got = wgb::expf_glibc(x);
        uint32_t a, b;
        memcpy(&a, &want, 4);
        memcpy(&b, &got, 4);
        checked++;
        if (a != b && !(std::isnan(want) && std::isnan(got))) {
            if (bad < 4) {
#pragma omp critical
                fprintf(stderr, "x=%a (0x%08x): libc %a, restated %a\n", x, u, want, got);
            }
            bad++;
        }
    }
    printf("checked %llu differ %llu\n", checked, bad);
    return bad != 0;
}
