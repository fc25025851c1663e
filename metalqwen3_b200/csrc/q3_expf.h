/*
 * q3_expf.h -- binary32 exp that returns the same bits as the host C library's
 * expf, usable from host C/C++ and from CUDA device code.
 *
 * Why: the reference computes SwiGLU (src/cpu/qwen3_original.c:450) and softmax
 * (:301) with the host libm's expf.  glibc's expf is not correctly rounded
 * (about 1.7e5 binary32 inputs differ from the correctly rounded result), so
 * bit-exact SwiGLU -> Q8_0 codes need the same function, not merely an accurate
 * one.
 *
 * Method (published as the "exp2f/expf with a 2^(i/N) table" method of
 * Szabolcs Nagy, ARM optimized-routines, used by glibc since 2.27): write
 * x*N/ln2 = k + r with N = 32, k integer (ties to even via the 1.5*2^52 shift)
 * and |r| <= 1/2; then exp(x) = 2^(k/N) * 2^(r/N), where 2^(k/N) is the table
 * entry 2^((k mod N)/N) with k/N added to its exponent field, and
 * 2^(r/N) ~= 1 + C2*r + C1*r^2 + C0*r^3 evaluated in binary64, rounded once to
 * binary32 at the end.  The table holds 2^(i/32) rounded to nearest binary64
 * (computed from the mathematics by gen_exp_table.py) with (i << 47) taken off
 * the bit pattern.  The host library on x86-64 selects its FMA build, so the
 * reduction x*N/ln2 and the polynomial use fused multiply-adds; this file
 * spells every FMA explicitly (and must be compiled without contraction).
 *
 * Verification: tests/test_expf.py compares this function with the host expf
 * on all 2^32 binary32 inputs (0 mismatches) and the GPU build with the host
 * on a strided sweep; a mismatch fails the build's tests, not silently.
 */
#ifndef Q3_EXPF_H
#define Q3_EXPF_H

#include <stdint.h>

#if defined(__CUDACC__)
#define Q3_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#include <string.h>
#define Q3_HD static inline
#endif

/* 2^(i/32) rounded to nearest binary64, minus (i << 47) on the bit pattern. */
#define Q3_EXP2_TAB32_INIT {                                                   \
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL,       \
    0x3fef9301d0125b51ULL, 0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL,       \
    0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL, 0x3fef06fe0a31b715ULL,       \
    0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,       \
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL,       \
    0x3feea47eb03a5585ULL, 0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL,       \
    0x3feea11473eb0187ULL, 0x3feea589994cce13ULL, 0x3feeace5422aa0dbULL,       \
    0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,       \
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL,       \
    0x3fef3720dcef9069ULL, 0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL,       \
    0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL }

/* Constants of the method: N/ln2, the rounding shift 1.5*2^52, and the
 * polynomial for 2^(r/N) scaled by N^-3, N^-2, N^-1. */
#define Q3_EXP_INVLN2N 0x1.71547652b82fep+5
#define Q3_EXP_SHIFT   0x1.8p+52
#define Q3_EXP_C0      0x1.c6af84b912394p-20
#define Q3_EXP_C1      0x1.ebfce50fac4f3p-13
#define Q3_EXP_C2      0x1.62e42ff0c52d6p-6

#if defined(__CUDACC__)
Q3_HD uint32_t q3_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}
Q3_HD uint64_t q3_d2u(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u; memcpy(&u, &d, 8); return u;
#endif
}
Q3_HD double q3_u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d; memcpy(&d, &u, 8); return d;
#endif
}
#define Q3_FMA(a, b, c) fma((a), (b), (c))
#else
Q3_HD uint32_t q3_f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
Q3_HD uint64_t q3_d2u(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }
Q3_HD double q3_u2d(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
#define Q3_FMA(a, b, c) fma((a), (b), (c))
#endif

/* `tab` is the 32-entry table above (in shared memory on the device). */
Q3_HD float q3_expf_tab(float x, const uint64_t *tab) {
    uint32_t ux = q3_f2u(x);
    uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                        /* |x| >= 88 or x is NaN/inf */
        if (ux == 0xff800000u) return 0.0f;        /* -inf */
        if (abstop >= 0x7f8u) return x + x;        /* +inf or NaN */
        if (x > 0x1.62e42ep6f) return (float)(Q3_EXP_SHIFT * Q3_EXP_SHIFT * Q3_EXP_SHIFT);  /* overflow: +inf */
        if (x < -0x1.9fe368p6f) return 0.0f;       /* underflow below 2^-150 */
    }
    double xd = (double)x;
    double kd = Q3_FMA(Q3_EXP_INVLN2N, xd, Q3_EXP_SHIFT);
    uint64_t ki = q3_d2u(kd);
    kd -= Q3_EXP_SHIFT;
    double r = Q3_FMA(Q3_EXP_INVLN2N, xd, -kd);
    uint64_t t = tab[ki & 31u] + (ki << 47);
    double s = q3_u2d(t);
    double z = Q3_FMA(Q3_EXP_C0, r, Q3_EXP_C1);
    double r2 = r * r;
    double y = Q3_FMA(Q3_EXP_C2, r, 1.0);
    y = Q3_FMA(z, r2, y);
    y = y * s;
    return (float)y;
}

/* ---------------------------------------------------------------------------
 * q3_expf_fast: the same function with the table read as separate high/low
 * 32-bit words (on the device: no shared-memory bank conflicts between lanes),
 * k/N added to the high word's exponent field, and the 64-bit integer add
 * avoided.  tests/test_expf.py checks it against the host expf on all 2^32
 * inputs as well.
 * ------------------------------------------------------------------------- */
#if defined(__CUDACC__)
Q3_HD double q3_hilo(uint32_t hi, uint32_t lo) {
#if defined(__CUDA_ARCH__)
    return __hiloint2double((int)hi, (int)lo);
#else
    return q3_u2d(((uint64_t)hi << 32) | lo);
#endif
}
Q3_HD uint32_t q3_dlo(double d) {
#if defined(__CUDA_ARCH__)
    return (uint32_t)__double2loint(d);
#else
    return (uint32_t)q3_d2u(d);
#endif
}
#else
Q3_HD double q3_hilo(uint32_t hi, uint32_t lo) { return q3_u2d(((uint64_t)hi << 32) | lo); }
Q3_HD uint32_t q3_dlo(double d) { return (uint32_t)q3_d2u(d); }
#endif

/* Inputs the core below does not cover: |x| >= 88, NaN, +-inf. */
Q3_HD int q3_expf_special(float x) { return ((q3_f2u(x) >> 20) & 0x7ffu) >= 0x42bu; }

/* The method's main path, valid when !q3_expf_special(x).  Branch-free, so a
 * kernel can evaluate it for every element and patch the rare special inputs
 * afterwards (for those it returns an unspecified finite or NaN value). */
Q3_HD float q3_expf_core(float x, const uint32_t *tab_hi, const uint32_t *tab_lo);

Q3_HD float q3_expf_fast(float x, const uint32_t *tab_hi, const uint32_t *tab_lo) {
    uint32_t ux = q3_f2u(x);
    if (q3_expf_special(x)) {                      /* |x| >= 88 or x is NaN/inf */
        if (ux == 0xff800000u) return 0.0f;
        if (((ux >> 20) & 0x7ffu) >= 0x7f8u) return x + x;
        if (x > 0x1.62e42ep6f) return (float)(Q3_EXP_SHIFT * Q3_EXP_SHIFT * Q3_EXP_SHIFT);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    return q3_expf_core(x, tab_hi, tab_lo);
}

Q3_HD float q3_expf_core(float x, const uint32_t *tab_hi, const uint32_t *tab_lo) {
    double xd = (double)x;
    double kd = Q3_FMA(Q3_EXP_INVLN2N, xd, Q3_EXP_SHIFT);
    uint32_t ki = q3_dlo(kd);
    kd -= Q3_EXP_SHIFT;
    double r = Q3_FMA(Q3_EXP_INVLN2N, xd, -kd);
    uint32_t j = ki & 31u;
    double s = q3_hilo(tab_hi[j] + (ki << 15), tab_lo[j]);   /* (ki << 47) reaches the high word only */
    double z = Q3_FMA(Q3_EXP_C0, r, Q3_EXP_C1);
    double r2 = r * r;
    double y = Q3_FMA(Q3_EXP_C2, r, 1.0);
    y = Q3_FMA(z, r2, y);
    y = y * s;
    return (float)y;
}

#endif /* Q3_EXPF_H */
