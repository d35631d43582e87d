/* Portable exponential for the sampler, identical on host and device.
 *
 * qs_exp_rn(x) returns exp(x) rounded to float, computed in IEEE double with
 * only +, *, fma, rint and exact power-of-two scaling, so the host (C) and
 * device (CUDA) builds return the same bits for every input:
 *   x = k*ln2 + r, |r| <= ln2/2 (Cody-Waite: ln2 = LN2_HI + LN2_LO, LN2_HI
 *   has 42 significant bits so k*LN2_HI is exact for |k| < 2^11);
 *   exp(r) by the Taylor series to r^13 (truncation < 5e-18 relative) in
 *   Horner form with fma; the double result is scaled by 2^k and rounded
 *   once to float.
 * The constants are ln 2 split as above, 1/ln 2 and 1/n!, each the double
 * nearest the exact value (derived with exact rational arithmetic).
 *
 * The reference sampler calls glibc's expf (sampler.h:197), whose result is
 * within 0.502 ulp and so differs from this correctly rounded value on a few
 * inputs; qs_exp_table.c records those inputs (measured by calling glibc's
 * expf on every float in [-110, 0]) and the device code applies them.
 */
#ifndef QS_EXP_H
#define QS_EXP_H

#ifdef __CUDACC__
#define QS_HD __host__ __device__ __forceinline__
#else
#define QS_HD static inline
#include <math.h>
#endif

#define QS_LN2_HI 0x1.62e42fefa3800p-1
#define QS_LN2_LO 0x1.ef35793c76730p-45
#define QS_INV_LN2 0x1.71547652b82fep+0

QS_HD float qs_exp_rn(float xf) {
    double x = (double)xf;
    if (!(x >= -150.0)) return (x != x) ? xf : 0.0f; /* NaN passes through; -inf / underflow -> 0 */
    if (x > 89.0) return (float)INFINITY;
    double k = rint(x * QS_INV_LN2);
    double r = fma(-k, QS_LN2_HI, x);
    r = fma(-k, QS_LN2_LO, r);
    double p = 0x1.6124613a86d09p-33;           /* 1/13! */
    p = fma(p, r, 0x1.1eed8eff8d898p-29);        /* 1/12! */
    p = fma(p, r, 0x1.ae64567f544e4p-26);        /* 1/11! */
    p = fma(p, r, 0x1.27e4fb7789f5cp-22);        /* 1/10! */
    p = fma(p, r, 0x1.71de3a556c734p-19);        /* 1/9!  */
    p = fma(p, r, 0x1.a01a01a01a01ap-16);        /* 1/8!  */
    p = fma(p, r, 0x1.a01a01a01a01ap-13);        /* 1/7!  */
    p = fma(p, r, 0x1.6c16c16c16c17p-10);        /* 1/6!  */
    p = fma(p, r, 0x1.1111111111111p-7);         /* 1/5!  */
    p = fma(p, r, 0x1.5555555555555p-5);         /* 1/4!  */
    p = fma(p, r, 0x1.5555555555555p-3);         /* 1/3!  */
    p = fma(p, r, 0x1.0000000000000p-1);         /* 1/2!  */
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
#ifdef __CUDA_ARCH__
    /* k is in [-217, 129] here and p in (0.7, 1.5), so p * 2^k is a normal
     * double and the product by the power of two built from its bits is
     * exact: the same value ldexp returns, without its general-case code. */
    return (float)(p * __longlong_as_double((long long)((int)k + 1023) << 52));
#else
    return (float)ldexp(p, (int)k);
#endif
}

#endif
