/* math_check.c -- exhaustive CPU checks of qwenium_b200/csrc/qs_math.h,
 * driven by tests/test_math_exhaustive.py.
 *
 *   math_check expf  <part> <nparts>   qs_expf == glibc expf, x in [-104, -0]
 *   math_check tanh  <part> <nparts>   qs_tanhf == (float)tanhl, x >= +0
 *   math_check tanhx <part> <nparts>   list tanh mismatches as "bits result"
 *   math_check runadd <seed> <cases>    qs_run_add == the sequential float loop
 *   math_check expftab <part> <nparts>  qs_expf_tab == qs_expf, x in [-104, -0]
 *   math_check scale <part> <nparts>    qs_fixed40 and qs_kround == their float
 *                                       definitions, t in [0, 1]
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
    } else if (!strcmp(what, "expftab")) {
        const uint64_t lo = 0x80000000u, hi = 0xC2D00000u; /* -0 .. -104 */
        const uint64_t n = hi - lo + 1, a = lo + n * part / nparts, b = lo + n * (part + 1) / nparts;
        for (uint64_t u = a; u < b; ++u) {
            float x;
            uint32_t w = (uint32_t)u;
            memcpy(&x, &w, 4);
            const float g = qs_expf(x), m = qs_expf_tab(x, qs_tab_exp32_h);
            if (memcmp(&g, &m, 4)) {
                if (bad < 5) printf("mismatch x=%a qs_expf=%a tab=%a\n", x, g, m);
                ++bad;
            }
        }
        if (qs_expf_tab(-INFINITY, qs_tab_exp32_h) != 0.0f) ++bad;
    } else if (!strcmp(what, "scale")) {
        static const int gs[] = {-20, -5, 0, 1, 3, 7, 12, 23};
        const uint64_t lo = 0u, hi = 0x3f800000u; /* +0 .. 1 */
        const uint64_t n = hi - lo + 1, a = lo + n * part / nparts, b = lo + n * (part + 1) / nparts;
        for (uint64_t u = a; u < b; ++u) {
            float t;
            uint32_t w = (uint32_t)u;
            memcpy(&t, &w, 4);
            if ((uint64_t)((double)t * 1099511627776.0) != qs_fixed40(t)) {
                if (bad < 5) printf("fixed40 mismatch t=%a\n", t);
                ++bad;
            }
            for (int j = 0; j < 8; ++j) {
                const float y = t * ldexpf(1.0f, 23 - gs[j]);
                int tie, big;
                const uint32_t k = qs_kround(t, gs[j], &tie, &big);
                if (y >= 16777216.0f) {
                    if (!big) ++bad;
                    continue;
                }
                if (big || k != (uint32_t)rintf(y) || tie != ((y - floorf(y)) == 0.5f)) {
                    if (bad < 5) printf("kround mismatch t=%a g=%d: %u vs %.1f\n", t, gs[j], k, (double)y);
                    ++bad;
                }
            }
        }
    } else if (!strcmp(what, "runadd")) {
        /* random runs: S over many binades (mantissas near the binade edge
           too), terms from far below half an ulp up to S, exact ties
           (n + 1/2 ulp), counts up to 30000, random or infinite stops */
        uint64_t st = 0x9E3779B97F4A7C15ull * (part + 1);
#define RNG() (st ^= st << 13, st ^= st >> 7, st ^= st << 17, st)
        for (uint64_t cs = 0; cs < nparts; ++cs) {
            const int e = (int)(RNG() % 40) - 20;
            uint32_t mant = (uint32_t)(RNG() & 0x7fffffu);
            if (RNG() % 4 == 0) mant = 0x7fffffu - (uint32_t)(RNG() % 64);
            float S0;
            uint32_t sbits = ((uint32_t)(e + 127) << 23) | mant;
            memcpy(&S0, &sbits, 4);
            float t;
            const int kind = (int)(RNG() % 4);
            if (kind == 0) { /* an exact tie: (n + 1/2) ulp(S0) */
                const double ulp = ldexp(1.0, e - 23);
                const double n = (double)(RNG() % 4096);
                t = (float)((n + 0.5) * ulp);
            } else if (kind == 1) { /* a tie at half an ulp of a later binade */
                const double ulp = ldexp(1.0, e - 22 + (int)(RNG() % 3));
                t = (float)((double)(RNG() % 64) * ulp + 0.5 * ulp);
            } else {
                const double f = ldexp((double)(RNG() % 1000000 + 1) / 1e6, -(int)(RNG() % 40));
                t = (float)(S0 * f);
            }
            const long long c = (long long)(RNG() % 30000) + 1;
            float stop = INFINITY;
            if (RNG() % 2) stop = (float)(S0 * (1.0 + (double)(RNG() % 1000) / 100.0));
            float Sa = S0, Sb = S0;
            long long ia = c;
            for (long long q = 0; q < c; ++q) {
                Sa = Sa + t;
                if (Sa >= stop) { ia = q; break; }
            }
            const long long ib = qs_run_add(&Sb, t, c, stop);
            if (ia != ib || memcmp(&Sa, &Sb, 4)) {
                if (bad < 5) printf("mismatch S0=%a t=%a c=%lld stop=%a: loop (%lld, %a) run (%lld, %a)\n", S0, t, c, stop, ia, Sa, ib, Sb);
                ++bad;
            }
        }
#undef RNG
    } else if (!strcmp(what, "runaddd")) {
        /* qs_run_add_d against the sequential double loop: S over binades
           around 2^-30 .. 2^0 (the cumulative weights of a draw), terms from
           far below half an ulp up to S, exact ties, counts up to 30000,
           random or infinite stops (a uniform in [0, 1)) */
        uint64_t st = 0xC2B2AE3D27D4EB4Full * (part + 1);
#define RNG() (st ^= st << 13, st ^= st >> 7, st ^= st << 17, st)
        for (uint64_t cs = 0; cs < nparts; ++cs) {
            const int e = -(int)(RNG() % 31);
            uint64_t mant = RNG() & ((1ull << 52) - 1ull);
            if (RNG() % 4 == 0) mant = ((1ull << 52) - 1ull) - (RNG() % 64);
            double S0;
            uint64_t sbits = ((uint64_t)(e + 1023) << 52) | mant;
            memcpy(&S0, &sbits, 8);
            if (RNG() % 8 == 0) S0 = 0.0;
            double t;
            const int kind = (int)(RNG() % 4);
            const int es = S0 > 0.0 ? e : -30;
            if (kind == 0) { /* an exact tie: (n + 1/2) ulp(S0) */
                t = ((double)(RNG() % 4096) + 0.5) * ldexp(1.0, es - 52);
            } else if (kind == 1) { /* a tie at half an ulp of a later binade */
                const double ulp = ldexp(1.0, es - 51 + (int)(RNG() % 3));
                t = (double)(RNG() % 64) * ulp + 0.5 * ulp;
            } else {
                const double f = ldexp((double)(RNG() % 1000000 + 1) / 1e6, -(int)(RNG() % 40));
                t = (S0 > 0.0 ? S0 : ldexp(1.0, es)) * f * (1.0 + (double)(RNG() % 1000003) * 1e-13);
            }
            const long long c = (long long)(RNG() % 30000) + 1;
            double stop = INFINITY;
            if (RNG() % 2) stop = (double)(RNG() % ((1ull << 53) - 1)) * ldexp(1.0, -53);
            double Sa = S0, Sb = S0;
            long long ia = c;
            for (long long q = 0; q < c; ++q) {
                Sa = Sa + t;
                if (Sa >= stop) { ia = q; break; }
            }
            const long long ib = qs_run_add_d(&Sb, t, c, stop);
            if (ia != ib || memcmp(&Sa, &Sb, 8)) {
                if (bad < 5) printf("mismatch S0=%a t=%a c=%lld stop=%a: loop (%lld, %a) run (%lld, %a)\n", S0, t, c, stop, ia, Sa, ib, Sb);
                ++bad;
            }
        }
#undef RNG
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
