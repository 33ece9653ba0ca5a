/* math_check.c -- exhaustive CPU checks of qwenium_b200/csrc/qs_math.h,
 * driven by tests/test_math_exhaustive.py.
 *
 *   math_check expf  <part> <nparts>   qs_expf == glibc expf, x in [-104, -0]
 *   math_check tanh  <part> <nparts>   qs_tanhf == (float)tanhl, x >= +0
 *   math_check tanhx <part> <nparts>   list tanh mismatches as "bits result"
 *
 * Prints "bad=<n>" and exits 0; the driver compares the count.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../qwenium_b200/csrc/qs_math.h"

int main(int argc, char** argv) {
    if (argc < 4) return 2;
    const char* what = argv[1];
    const uint64_t part = (uint64_t)atoll(argv[2]), nparts = (uint64_t)atoll(argv[3]);
    long bad = 0;
    if (!strcmp(what, "expf")) {
        const uint64_t lo = 0x80000000u, hi = 0xC2D00000u; /* -0 .. -104 */
        const uint64_t n = hi - lo + 1, a = lo + n * part / nparts, b = lo + n * (part + 1) / nparts;
        for (uint64_t u = a; u < b; ++u) {
            float x;
            uint32_t w = (uint32_t)u;
            memcpy(&x, &w, 4);
            const float g = expf(x), m = qs_expf(x);
            if (memcmp(&g, &m, 4)) {
                if (bad < 5) printf("mismatch x=%a glibc=%a qs=%a\n", x, g, m);
                ++bad;
            }
        }
        /* -inf and the underflow edge */
        if (qs_expf(-INFINITY) != 0.0f) ++bad;
    } else if (!strcmp(what, "tanh") || !strcmp(what, "tanhx")) {
        const int list = !strcmp(what, "tanhx");
        const uint64_t lo = 0, hi = 0x7F800000u; /* +0 .. +inf */
        const uint64_t n = hi - lo + 1, a = lo + n * part / nparts, b = lo + n * (part + 1) / nparts;
        for (uint64_t u = a; u < b; ++u) {
            float x;
            uint32_t w = (uint32_t)u;
            memcpy(&x, &w, 4);
            const float ref = (float)tanhl((long double)x), m = qs_tanhf(x);
            const float mneg = qs_tanhf(-x);
            if (memcmp(&ref, &m, 4) || mneg != -ref) {
                uint32_t rb;
                memcpy(&rb, &ref, 4);
                if (list) printf("0x%08xu 0x%08xu\n", w, rb);
                else if (bad < 5) printf("mismatch x=%a tanhl=%a qs=%a\n", x, ref, m);
                ++bad;
            }
        }
    } else {
        return 2;
    }
    printf("bad=%ld\n", bad);
    return 0;
}
