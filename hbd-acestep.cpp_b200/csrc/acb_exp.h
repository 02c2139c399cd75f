/* acb_exp.h -- the exponential every softmax and SiLU of libacb uses, written once so that the
 * GPU kernels and any C program on the host compute bit-identical values.
 *
 * exp(x) = 2^k * exp(r): k = nearest integer to x*log2(e), r = x - k*ln2 by the Cody-Waite
 * two-constant reduction (W. J. Cody and W. Waite, Software Manual for the Elementary
 * Functions, 1980) with fused multiply-adds, exp(r) for |r| <= ln2/2 by its Taylor polynomial
 * of degree 8 in Horner form (truncation below 0.02 ulp), then the power of two applied in two
 * exact halves so that results down to the subnormal range round once. Every step is an IEEE
 * single-precision operation with one rounding (multiply, add, fused multiply-add, exponent-field
 * assembly), so the result depends on nothing but x: a C compiler that keeps
 * these operations separate (no contraction of the plain multiply) and a CUDA kernel give the
 * same bits. Accuracy: within 2 ulp of exp over the whole float range (checked in the tests
 * against a double-precision exp). NaN propagates, x > 88.72 gives +inf, x < -103.98 gives 0.
 *
 * Plain C99 / CUDA C++; include it from a .cu or a .c file. */
#ifndef ACB_EXP_H
#define ACB_EXP_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#    define ACB_EXP_FN static __host__ __device__ __forceinline__
#    if defined(__CUDA_ARCH__)
#        define ACB_EXP_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#        define ACB_EXP_MUL(a, b)    __fmul_rn((a), (b))
#        define ACB_EXP_ADD(a, b)    __fadd_rn((a), (b))
#    else
#        include <math.h>
#        define ACB_EXP_FMA(a, b, c) fmaf((a), (b), (c))
#        define ACB_EXP_MUL(a, b)    ((a) * (b))
#        define ACB_EXP_ADD(a, b)    ((a) + (b))
#    endif
#else
#    include <math.h>
#    define ACB_EXP_FN           static inline
#    define ACB_EXP_FMA(a, b, c) fmaf((a), (b), (c))
#    define ACB_EXP_MUL(a, b)    ((a) * (b))
#    define ACB_EXP_ADD(a, b)    ((a) + (b))
#endif

ACB_EXP_FN uint32_t acb_exp_bits(float f) {
    uint32_t u;
#if defined(__CUDA_ARCH__)
    u = __float_as_uint(f);
#else
    memcpy(&u, &f, 4);
#endif
    return u;
}

/* 2^e as a float for -126 <= e <= 127 (exponent field assembled directly: exact) */
ACB_EXP_FN float acb_exp_pow2i(int e) {
    uint32_t u = (uint32_t) (e + 127) << 23;
    float    f;
#if defined(__CUDA_ARCH__)
    f = __uint_as_float(u);
#else
    memcpy(&f, &u, 4);
#endif
    return f;
}

ACB_EXP_FN float acb_expf(float x) {
    if (x != x) {
        return x;
    }
    if (x > 88.7228394f) {
        return 1.0f / 0.0f;
    }
    if (x < -103.972084f) {
        return 0.0f;
    }
    /* k = rint(x / ln2) by the round-to-nearest-even of adding 1.5 * 2^23 (|x / ln2| < 2^22, so
     * the integer lands in the low mantissa bits: k's float value and its int value come out of
     * two plain additions, no conversion instruction); r = x - k ln2 (ln2 = LN2_HI + LN2_LO) */
    const float t = ACB_EXP_ADD(ACB_EXP_MUL(x, 1.44269502f), 12582912.0f);
    const float k = ACB_EXP_ADD(t, -12582912.0f);
    float       r = ACB_EXP_FMA(k, -0.693145751953125f, x);
    r             = ACB_EXP_FMA(k, -1.42860677e-06f, r);
    /* sum_{n<=8} r^n / n! */
    float p = 2.48015873e-05f;           /* 1/8! */
    p       = ACB_EXP_FMA(p, r, 1.98412698e-04f); /* 1/7! */
    p       = ACB_EXP_FMA(p, r, 1.38888889e-03f); /* 1/6! */
    p       = ACB_EXP_FMA(p, r, 8.33333377e-03f); /* 1/5! */
    p       = ACB_EXP_FMA(p, r, 4.16666679e-02f); /* 1/4! */
    p       = ACB_EXP_FMA(p, r, 1.66666672e-01f); /* 1/3! */
    p       = ACB_EXP_FMA(p, r, 0.5f);
    p       = ACB_EXP_FMA(p, r, 1.0f);
    p       = ACB_EXP_FMA(p, r, 1.0f);
    /* p * 2^k, k in [-150, 128]: two factors 2^(k/2) and 2^(k - k/2), each a normal float; the
     * first product is exact, the second rounds once (into the subnormals when it must) */
    const int ki = (int) (acb_exp_bits(t) - 0x4B400000u);
    const int k1 = ki / 2;
    return ACB_EXP_MUL(ACB_EXP_MUL(p, acb_exp_pow2i(k1)), acb_exp_pow2i(ki - k1));
}

#endif
