// qs_math.h -- deterministic scalar math shared by the CUDA kernels and by the
// CPU tests that pin it. Every double operation is an explicit, separately
// rounded IEEE operation (device: __dmul_rn/__dadd_rn/__fma_rn intrinsics,
// which nvcc never contracts; host: plain operators under -ffp-contract=off),
// so a host build and a device build produce identical bits.
//
//   qs_expf(x)  -- the float exponential exactly as glibc 2.39 computes it on
//                  x86-64 with FMA (the library the reference's
//                  `expf(p.second - max_l)` calls, src/sampling/sampling.cpp
//                  :171,175,186). Restates the published algorithm of glibc's
//                  sysdeps/ieee754/flt-32/e_expf.c (from ARM's
//                  optimized-routines): z = x*32/ln2, k = round(z),
//                  r = z - k, 2^(r/32) by a cubic in double, scaled by a
//                  32-entry table of 2^(i/32); the result rounded to float.
//                  The table below is 2^(i/32) rounded to nearest (computed
//                  from the definition). tests/test_math_exhaustive.py checks
//                  qs_expf == expf for every float in [-104, 0].
//   qs_tanhf(y) -- correctly rounded float tanh, for the soft-cap
//                  cap*tanh(x/cap) (ggml's build_softcap, reference
//                  layers/attention.cpp:30-36). Evaluated as em/(em+2) with
//                  em = expm1(2|y|) in double (table 2^(j/64) in hi+lo parts,
//                  degree-6 Taylor polynomial). Equal to (float)tanhl on all
//                  2^32 float inputs (tests/test_math_exhaustive.py).
#ifndef QS_MATH_H
#define QS_MATH_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define QS_HD __host__ __device__ __forceinline__
#define QS_CONST __device__ __constant__
#else
#define QS_HD static inline
#define QS_CONST static const
#endif

#if defined(__CUDA_ARCH__)
#define QS_DMUL(a, b) __dmul_rn((a), (b))
#define QS_DADD(a, b) __dadd_rn((a), (b))
#define QS_DSUB(a, b) __dsub_rn((a), (b))
#define QS_DFMA(a, b, c) __fma_rn((a), (b), (c))
#define QS_DDIV(a, b) __ddiv_rn((a), (b))
#define QS_D2F(a) __double2float_rn(a)
#define QS_FADD(a, b) __fadd_rn((a), (b))
#define QS_TAB_EXP32 qs_tab_exp32_d
#define QS_TAB_EXP64_HI qs_tab_exp64_hi_d
#define QS_TAB_EXP64_LO qs_tab_exp64_lo_d
#else
#include <math.h>
#define QS_DMUL(a, b) ((a) * (b))
#define QS_DADD(a, b) ((a) + (b))
#define QS_DSUB(a, b) ((a) - (b))
#define QS_DFMA(a, b, c) fma((a), (b), (c))
#define QS_DDIV(a, b) ((a) / (b))
#define QS_D2F(a) ((float)(a))
#define QS_FADD(a, b) ((a) + (b))
#define QS_TAB_EXP32 qs_tab_exp32_h
#define QS_TAB_EXP64_HI qs_tab_exp64_hi_h
#define QS_TAB_EXP64_LO qs_tab_exp64_lo_h
#endif

QS_HD uint32_t qs_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}
QS_HD float qs_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}
QS_HD uint64_t qs_d2u(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u;
    memcpy(&u, &d, 8);
    return u;
#endif
}
QS_HD double qs_u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d;
    memcpy(&d, &u, 8);
    return d;
#endif
}

// ---- tables (values derived from their definitions, see header) ----------
// bits(2^(i/32)) - (i << 47): adding k << 47 for k = 32*e + i yields
// bits(2^e * 2^(i/32)).
#define QS_EXP32_TABLE                                                                  \
    {0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL, \
     0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL, \
     0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL, \
     0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL, \
     0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL, \
     0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL, \
     0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL, \
     0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL}

// 2^(j/64) = hi + lo, hi rounded to nearest double, lo the remainder.
#define QS_EXP64_HI_TABLE                                                                          \
    {0x1.0000000000000p+0, 0x1.02c9a3e778061p+0, 0x1.059b0d3158574p+0, 0x1.0874518759bc8p+0,     \
     0x1.0b5586cf9890fp+0, 0x1.0e3ec32d3d1a2p+0, 0x1.11301d0125b51p+0, 0x1.1429aaea92de0p+0,     \
     0x1.172b83c7d517bp+0, 0x1.1a35beb6fcb75p+0, 0x1.1d4873168b9aap+0, 0x1.2063b88628cd6p+0,     \
     0x1.2387a6e756238p+0, 0x1.26b4565e27cddp+0, 0x1.29e9df51fdee1p+0, 0x1.2d285a6e4030bp+0,     \
     0x1.306fe0a31b715p+0, 0x1.33c08b26416ffp+0, 0x1.371a7373aa9cbp+0, 0x1.3a7db34e59ff7p+0,     \
     0x1.3dea64c123422p+0, 0x1.4160a21f72e2ap+0, 0x1.44e086061892dp+0, 0x1.486a2b5c13cd0p+0,     \
     0x1.4bfdad5362a27p+0, 0x1.4f9b2769d2ca7p+0, 0x1.5342b569d4f82p+0, 0x1.56f4736b527dap+0,     \
     0x1.5ab07dd485429p+0, 0x1.5e76f15ad2148p+0, 0x1.6247eb03a5585p+0, 0x1.6623882552225p+0,     \
     0x1.6a09e667f3bcdp+0, 0x1.6dfb23c651a2fp+0, 0x1.71f75e8ec5f74p+0, 0x1.75feb564267c9p+0,     \
     0x1.7a11473eb0187p+0, 0x1.7e2f336cf4e62p+0, 0x1.82589994cce13p+0, 0x1.868d99b4492edp+0,     \
     0x1.8ace5422aa0dbp+0, 0x1.8f1ae99157736p+0, 0x1.93737b0cdc5e5p+0, 0x1.97d829fde4e50p+0,     \
     0x1.9c49182a3f090p+0, 0x1.a0c667b5de565p+0, 0x1.a5503b23e255dp+0, 0x1.a9e6b5579fdbfp+0,     \
     0x1.ae89f995ad3adp+0, 0x1.b33a2b84f15fbp+0, 0x1.b7f76f2fb5e47p+0, 0x1.bcc1e904bc1d2p+0,     \
     0x1.c199bdd85529cp+0, 0x1.c67f12e57d14bp+0, 0x1.cb720dcef9069p+0, 0x1.d072d4a07897cp+0,     \
     0x1.d5818dcfba487p+0, 0x1.da9e603db3285p+0, 0x1.dfc97337b9b5fp+0, 0x1.e502ee78b3ff6p+0,     \
     0x1.ea4afa2a490dap+0, 0x1.efa1bee615a27p+0, 0x1.f50765b6e4540p+0, 0x1.fa7c1819e90d8p+0}
#define QS_EXP64_LO_TABLE                                                                          \
    {0x0p+0, -0x1.19083535b085dp-56, 0x1.d73e2a475b465p-55, 0x1.186be4bb284ffp-57,               \
     0x1.8a62e4adc610bp-54, 0x1.03a1727c57b53p-59, -0x1.6c51039449b3ap-54, -0x1.32fbf9af1369ep-54, \
     -0x1.19041b9d78a76p-55, 0x1.e5b4c7b4968e4p-55, 0x1.e016e00a2643cp-54, 0x1.dc775814a8495p-55, \
     0x1.9b07eb6c70573p-54, 0x1.2bd339940e9d9p-55, 0x1.612e8afad1255p-55, 0x1.0024754db41d5p-54,   \
     0x1.6f46ad23182e4p-55, 0x1.32721843659a6p-54, -0x1.63aeabf42eae2p-54, -0x1.5e436d661f5e3p-56, \
     0x1.ada0911f09ebcp-55, -0x1.ef3691c309278p-58, 0x1.89b7a04ef80d0p-59, 0x1.3c1a3b69062f0p-56, \
     0x1.d4397afec42e2p-56, -0x1.4b309d25957e3p-54, -0x1.07abe1db13cadp-55, 0x1.9bb2c011d93adp-54, \
     0x1.6324c054647adp-54, 0x1.ba6f93080e65ep-54, -0x1.383c17e40b497p-54, -0x1.bb60987591c34p-54, \
     -0x1.bdd3413b26456p-54, -0x1.bbe3a683c88abp-57, -0x1.16e4786887a99p-55, -0x1.0245957316dd3p-54, \
     -0x1.41577ee04992fp-55, 0x1.05d02ba15797ep-56, -0x1.d4c1dd41532d8p-54, -0x1.fc6f89bd4f6bap-54, \
     0x1.6e9f156864b27p-54, 0x1.5cc13a2e3976cp-55, -0x1.75fc781b57ebcp-57, -0x1.d185b7c1b85d1p-54, \
     0x1.c7c46b071f2bep-56, -0x1.359495d1cd533p-54, -0x1.d2f6edb8d41e1p-54, 0x1.0fac90ef7fd31p-54, \
     0x1.7a1cd345dcc81p-54, -0x1.2805e3084d708p-57, -0x1.5584f7e54ac3bp-56, 0x1.23dd07a2d9e84p-55, \
     0x1.11065895048ddp-55, 0x1.2884dff483cadp-54, 0x1.503cbd1e949dbp-56, -0x1.cbc3743797a9cp-54, \
     0x1.2ed02d75b3707p-55, 0x1.c2300696db532p-54, -0x1.1a5cd4f184b5cp-54, 0x1.39e8980a9cc8fp-55, \
     -0x1.e9c23179c2893p-54, 0x1.dc7f486a4b6b0p-54, 0x1.9d3e12dd8a18bp-54, 0x1.74853f3a5931ep-55}

#if defined(__CUDACC__)
__device__ __constant__ uint64_t qs_tab_exp32_d[32] = QS_EXP32_TABLE;
__device__ __constant__ double qs_tab_exp64_hi_d[64] = QS_EXP64_HI_TABLE;
__device__ __constant__ double qs_tab_exp64_lo_d[64] = QS_EXP64_LO_TABLE;
#endif
#if !defined(__CUDA_ARCH__)
static const uint64_t qs_tab_exp32_h[32] = QS_EXP32_TABLE;
static const double qs_tab_exp64_hi_h[64] = QS_EXP64_HI_TABLE;
static const double qs_tab_exp64_lo_h[64] = QS_EXP64_LO_TABLE;
#endif

// ---- expf, as glibc 2.39 computes it --------------------------------------
// qs_expf_tab: the finite x <= 0 part of qs_expf (no NaN, infinity or
// overflow branches; x below the underflow edge, -inf included, gives 0) with
// the 2^(i/32) table passed in. Device code keeps a copy of the table in
// shared memory: lanes index it at random, which a __constant__ array
// serialises.
QS_HD float qs_expf_tab(float x, const uint64_t* tab) {
    if (x < -0x1.9fe368p6f) return 0.0f;               // below the smallest subnormal/2
    const double InvLn2N = 0x1.71547652b82fep+5;       // 32/ln2
    const double SHIFT = 0x1.8p+52;                    // round-to-integer shift
    const double C0 = 0x1.c6af84b912394p-20;           // cubic for 2^(r/32)
    const double C1 = 0x1.ebfce50fac4f3p-13;
    const double C2 = 0x1.62e42ff0c52d6p-6;
    const double xd = (double)x;
    const double z = QS_DMUL(InvLn2N, xd);
    double kd = QS_DADD(z, SHIFT);
    const uint64_t ki = qs_d2u(kd);
    kd = QS_DSUB(kd, SHIFT);
    const double r = QS_DFMA(InvLn2N, xd, -kd);
    uint64_t t = tab[ki % 32];
    t += ki << 47;
    const double s = qs_u2d(t);
    const double zz = QS_DFMA(C0, r, C1);
    const double r2 = QS_DMUL(r, r);
    double y = QS_DFMA(C2, r, 1.0);
    y = QS_DFMA(zz, r2, y);
    y = QS_DMUL(y, s);
    return QS_D2F(y);
}
QS_HD float qs_expf(float x) {
    if (x != x) return x + x;                          // NaN
    if (x == -__builtin_huge_valf()) return 0.0f;
    if (x > 0x1.62e42ep6f) return __builtin_huge_valf();
    return qs_expf_tab(x, QS_TAB_EXP32);
}

// ---- exact scalings of a float, by integer arithmetic ----------------------
// qs_fixed40(t) = (uint64)(t * 2^40) truncated, for 0 <= t <= 1 (t * 2^40 is
// exact in double; the conversion truncates).
QS_HD uint64_t qs_fixed40(float t) {
    const uint32_t u = qs_f2u(t);
    const int e = (int)(u >> 23);
    const uint64_t mt = (uint64_t)((u & 0x7fffffu) | 0x800000u);
    return e >= 110 ? mt << (e - 110) : (e > 86 ? mt >> (110 - e) : 0u);
}
// qs_kround(p, g) = rintf(p * 2^(23-g)) (round half to even) for p >= 0
// while that is below 2^24; *tie: p * 2^(23-g) is exactly half-way between
// integers; *big: it is 2^24 or more (the result is then 0).
QS_HD uint32_t qs_kround(float p, int g, int* tie, int* big) {
    const uint32_t u = qs_f2u(p);
    int e = (int)(u >> 23);
    uint32_t mt = u & 0x7fffffu;
    if (e) mt |= 0x800000u;
    else e = 1;                                        // subnormal
    const int q = e - 127 - g;                         // p * 2^(23-g) = mt * 2^q
    *tie = 0;
    *big = q > 0;
    if (q >= 0) return q > 0 ? 0u : mt;
    if (q <= -25) return 0u;                           // below 1/2
    const int sh = -q;
    const uint32_t fl = mt >> sh, rem = mt & ((1u << sh) - 1u), half = 1u << (sh - 1);
    *tie = rem == half;
    return fl + ((rem > half || (rem == half && (fl & 1u))) ? 1u : 0u);
}

// ---- expm1(z) for 2^-12 <= z <= 19, about 1 ulp (double) ------------------
QS_HD double qs_expm1_pos(double z) {
    const double InvL = 0x1.71547652b82fep+6;          // 64/ln2
    const double Lhi = 0x1.62e4200000000p-7;           // ln2/64, 32 trailing zero bits
    const double Llo = 0x1.fdf473de6af28p-28;
    const double SHIFT = 0x1.8p+52;
    double nd = QS_DADD(QS_DMUL(z, InvL), SHIFT);
    const int64_t n = (int64_t)(qs_d2u(nd) & 0xFFFFFFFFULL);  // 0 <= n < 2^32
    nd = QS_DSUB(nd, SHIFT);
    double r = QS_DFMA(-nd, Lhi, z);
    r = QS_DFMA(-nd, Llo, r);
    const int j = (int)(n & 63);
    const int k = (int)(n >> 6);
    // p = e^r - 1 = r + r^2/2 + ... + r^6/720
    double p = QS_DFMA(r, 0x1.6c16c16c16c17p-10, 0x1.1111111111111p-7);
    p = QS_DFMA(r, p, 0x1.5555555555555p-5);
    p = QS_DFMA(r, p, 0x1.5555555555555p-3);
    p = QS_DFMA(r, p, 0x1.0p-1);
    p = QS_DFMA(r, p, 1.0);
    p = QS_DMUL(r, p);
    const double th = QS_TAB_EXP64_HI[j], tl = QS_TAB_EXP64_LO[j];
    const double sc = qs_u2d((uint64_t)(1023 + k) << 52);  // 2^k, exact
    // e^z - 1 = (2^k*th - 1) + 2^k*(th*p + tl*(1+p)); the first term is exact.
    const double a = QS_DSUB(QS_DMUL(sc, th), 1.0);
    const double c = QS_DFMA(th, p, QS_DFMA(tl, p, tl));
    return QS_DFMA(sc, c, a);
}

QS_HD float qs_tanhf(float y) {
    if (y != y) return y + y;
    const uint32_t ub = qs_f2u(y);
    const uint32_t sign = ub & 0x80000000u;
    const uint32_t ab = ub & 0x7fffffffu;
    const float a = qs_u2f(ab);
    float r;
    if (a < 0x1.0p-12f) {
        r = a;                                          // |tanh(a) - a| < ulp(a)/2
    } else if (a >= 9.1f) {
        r = 1.0f;                                       // 1 - tanh(a) < 2^-25
    } else {
        const double em = qs_expm1_pos(QS_DMUL(2.0, (double)a));
        r = QS_D2F(QS_DDIV(em, QS_DADD(em, 2.0)));
    }
    return qs_u2f(qs_f2u(r) | sign);
}

// ggml's build_softcap on one value: scale by (1/cap), tanh, scale by cap.
QS_HD float qs_softcap(float x, float cap) {
#if defined(__CUDA_ARCH__)
    const float inv = __fdiv_rn(1.0f, cap);
    return __fmul_rn(cap, qs_tanhf(__fmul_rn(x, inv)));
#else
    const float inv = 1.0f / cap;
    return cap * qs_tanhf(x * inv);
#endif
}

// Order-preserving uint32 key of a float (larger float -> larger key). NaNs
// are mapped to -inf by the callers before keying.
QS_HD uint32_t qs_key(float f) {
    const uint32_t u = qs_f2u(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
QS_HD float qs_unkey(uint32_t k) {
    return qs_u2f((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

QS_HD float qs_bf16_to_f32(uint16_t b) { return qs_u2f((uint32_t)b << 16); }

// qs_run_add: c sequential float additions of the same term,
//     for (i = 0; i < c; ++i) { S = S + t; if (S >= stop) return i; }  return c;
// (round to nearest, ties to even) in O(1) per binade of S instead of O(c).
// While the exact sum stays in S's binade [2^e, 2^(e+1)), S + t rounds to
// S + rne(t / ulp) * ulp, so a run of equal terms adds a constant integer
// k = rne(t / ulp) ulps -- except that when t / ulp is a half-integer n + 1/2
// the rounding goes to the even neighbour: once S's mantissa is even every
// add contributes n + (n & 1); an odd mantissa takes one single step first.
// The add that leaves the binade, and operands outside the normal range, are
// done as real float additions. Integer arithmetic on the encodings only, so
// host and device agree bit for bit. S >= 0, t >= 0, stop >= 0 (or +inf).
QS_HD long long qs_run_add(float* Sp, float t, long long c, float stop) {
    float S = *Sp;
    long long i = 0;
    const uint32_t tb = qs_f2u(t);
    const int et = (int)((tb >> 23) & 0xffu);
    const uint64_t mt = et ? (uint64_t)((tb & 0x7fffffu) | 0x800000u) : (uint64_t)(tb & 0x7fffffu);
    const int Et = (et ? et : 1) - 150;  /* t = mt * 2^Et */
    const uint32_t pb = qs_f2u(stop);
    const int stop_inf = ((pb >> 23) & 0xffu) == 0xffu;
    const int ep = (int)((pb >> 23) & 0xffu);
    const uint64_t mp = ep ? (uint64_t)((pb & 0x7fffffu) | 0x800000u) : (uint64_t)(pb & 0x7fffffu);
    const int Ep = (ep ? ep : 1) - 150;  /* stop = mp * 2^Ep */
    const uint64_t lim = 1ull << 24;
    while (i < c) {
        const uint32_t sb = qs_f2u(S);
        const int es = (int)((sb >> 23) & 0xffu);
        if (es == 0 || es >= 253 || tb == 0u) {
            /* S zero or subnormal, near overflow, or t == 0: real adds (t == 0
               leaves S unchanged: the first add decides) */
            S = QS_FADD(S, t);
            if (S >= stop) { *Sp = S; return i; }
            ++i;
            if (tb == 0u) { *Sp = S; return c; }
            continue;
        }
        const uint64_t ms = (uint64_t)((sb & 0x7fffffu) | 0x800000u);
        const int Es = es - 150; /* S = ms * 2^Es, ulp = 2^Es */
        const int d = Es - Et;    /* t / ulp = mt * 2^-d */
        uint64_t k;
        int tie = 0;
        uint64_t n;
        if (d <= 0) {
            if (-d >= 40) { S = QS_FADD(S, t); if (S >= stop) { *Sp = S; return i; } ++i; continue; }
            n = mt << (-d);
            k = n;
        } else if (d >= 40) {
            n = 0;
            k = 0; /* t < 2^-16 ulp */
        } else {
            n = mt >> d;
            const uint64_t rem = mt & ((1ull << d) - 1ull), half = 1ull << (d - 1);
            tie = rem == half;
            k = n + (rem > half ? 1u : 0u);
        }
        if (tie && (ms & 1u)) {
            /* one step to an even mantissa */
            const uint64_t r = ms + n + ((ms + n) & 1u);
            if (r > lim) { S = QS_FADD(S, t); if (S >= stop) { *Sp = S; return i; } ++i; continue; }
            S = r == lim ? qs_u2f((uint32_t)(es + 1) << 23) : qs_u2f(((uint32_t)es << 23) | (uint32_t)(r - 0x800000u));
            if (S >= stop) { *Sp = S; return i; }
            ++i;
            continue;
        }
        if (tie) k = n + (n & 1u);
        if (k == 0) { /* S never changes again */
            *Sp = S;
            return (S >= stop) ? i : c;
        }
        const uint64_t room = (lim - ms) / k;
        if (room == 0) { /* the next add leaves the binade */
            S = QS_FADD(S, t);
            if (S >= stop) { *Sp = S; return i; }
            ++i;
            continue;
        }
        const uint64_t left = (uint64_t)(c - i);
        const uint64_t nadd = room < left ? room : left;
        if (!stop_inf) {
            /* first j >= 1 with (ms + j k) 2^Es >= mp 2^Ep */
            const int D2 = Ep - Es;
            uint64_t T;
            int never = 0;
            if (D2 >= 0) {
                if (D2 >= 40 || (mp << D2) > (1ull << 50)) never = 1;
                T = never ? 0 : (mp << D2);
            } else {
                const int sh = -D2;
                T = sh >= 63 ? (mp ? 1u : 0u) : ((mp + (1ull << sh) - 1ull) >> sh);
            }
            if (!never) {
                const uint64_t j = T <= ms ? 1u : (T - ms + k - 1u) / k;
                if (j <= nadd) {
                    const uint64_t r = ms + j * k;
                    S = r == lim ? qs_u2f((uint32_t)(es + 1) << 23) : qs_u2f(((uint32_t)es << 23) | (uint32_t)(r - 0x800000u));
                    *Sp = S;
                    return i + (long long)j - 1;
                }
            }
        }
        const uint64_t r = ms + nadd * k;
        S = r == lim ? qs_u2f((uint32_t)(es + 1) << 23) : qs_u2f(((uint32_t)es << 23) | (uint32_t)(r - 0x800000u));
        i += (long long)nadd;
    }
    *Sp = S;
    return c;
}

// qs_run_add_d: qs_run_add for doubles (53-bit significands),
//     for (i = 0; i < c; ++i) { S = S + t; if (S >= stop) return i; }  return c;
// with the same per-binade identity: while the exact sum stays in S's binade
// every add contributes k = rne(t / ulp) ulps (a half-integer t / ulp rounds
// to the even neighbour), so a run takes O(1) per binade. The draw of
// std::discrete_distribution accumulates its cumulative weights this way in
// double (libstdc++'s partial_sum). S >= 0, t >= 0, stop >= 0 (or +inf).
QS_HD long long qs_run_add_d(double* Sp, double t, long long c, double stop) {
    double S = *Sp;
    long long i = 0;
    const uint64_t M52 = (1ull << 52) - 1ull;
    const uint64_t tb = qs_d2u(t);
    const int et = (int)((tb >> 52) & 0x7ffu);
    const uint64_t mt = et ? ((tb & M52) | (1ull << 52)) : (tb & M52);
    const int Et = (et ? et : 1) - 1075; /* t = mt * 2^Et */
    const uint64_t pb = qs_d2u(stop);
    const int stop_inf = ((pb >> 52) & 0x7ffu) == 0x7ffu;
    const int ep = (int)((pb >> 52) & 0x7ffu);
    const uint64_t mp = ep ? ((pb & M52) | (1ull << 52)) : (pb & M52);
    const int Ep = (ep ? ep : 1) - 1075; /* stop = mp * 2^Ep */
    const uint64_t lim = 1ull << 53;
    while (i < c) {
        const uint64_t sb = qs_d2u(S);
        const int es = (int)((sb >> 52) & 0x7ffu);
        if (es == 0 || es >= 2045 || tb == 0u) {
            S = QS_DADD(S, t);
            if (S >= stop) { *Sp = S; return i; }
            ++i;
            if (tb == 0u) { *Sp = S; return c; }
            continue;
        }
        const uint64_t ms = (sb & M52) | (1ull << 52);
        const int Es = es - 1075; /* S = ms * 2^Es, ulp = 2^Es */
        const int d = Es - Et;    /* t / ulp = mt * 2^-d */
        uint64_t k, n;
        int tie = 0;
        if (d <= 0) {
            if (-d >= 11) { S = QS_DADD(S, t); if (S >= stop) { *Sp = S; return i; } ++i; continue; }
            n = mt << (-d);
            k = n;
        } else if (d >= 64) {
            n = 0;
            k = 0; /* t < 2^-11 ulp */
        } else {
            n = mt >> d;
            const uint64_t rem = mt & ((1ull << d) - 1ull), half = 1ull << (d - 1);
            tie = rem == half;
            k = n + (rem > half ? 1u : 0u);
        }
        if (tie && (ms & 1u)) {
            const uint64_t r = ms + n + ((ms + n) & 1u);
            if (r > lim) { S = QS_DADD(S, t); if (S >= stop) { *Sp = S; return i; } ++i; continue; }
            S = r == lim ? qs_u2d((uint64_t)(es + 1) << 52) : qs_u2d(((uint64_t)es << 52) | (r - (1ull << 52)));
            if (S >= stop) { *Sp = S; return i; }
            ++i;
            continue;
        }
        if (tie) k = n + (n & 1u);
        if (k == 0) {
            *Sp = S;
            return (S >= stop) ? i : c;
        }
        const uint64_t room = (lim - ms) / k;
        if (room == 0) {
            S = QS_DADD(S, t);
            if (S >= stop) { *Sp = S; return i; }
            ++i;
            continue;
        }
        const uint64_t left = (uint64_t)(c - i);
        const uint64_t nadd = room < left ? room : left;
        if (!stop_inf) {
            const int D2 = Ep - Es;
            uint64_t T;
            int never = 0;
            if (D2 >= 0) {
                if (D2 >= 11 || (mp << D2) > (1ull << 62)) never = 1;
                T = never ? 0 : (mp << D2);
            } else {
                const int sh = -D2;
                T = sh >= 63 ? (mp ? 1u : 0u) : ((mp + (1ull << sh) - 1ull) >> sh);
            }
            if (!never) {
                const uint64_t j = T <= ms ? 1u : (T - ms + k - 1u) / k;
                if (j <= nadd) {
                    const uint64_t r = ms + j * k;
                    S = r == lim ? qs_u2d((uint64_t)(es + 1) << 52) : qs_u2d(((uint64_t)es << 52) | (r - (1ull << 52)));
                    *Sp = S;
                    return i + (long long)j - 1;
                }
            }
        }
        const uint64_t r = ms + nadd * k;
        S = r == lim ? qs_u2d((uint64_t)(es + 1) << 52) : qs_u2d(((uint64_t)es << 52) | (r - (1ull << 52)));
        i += (long long)nadd;
    }
    *Sp = S;
    return c;
}

#endif  // QS_MATH_H
