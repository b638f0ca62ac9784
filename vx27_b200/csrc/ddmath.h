// Correctly rounded double-precision exp and log for the DeltaNet gate mapping.
//
// The reference computes its gates on the host in double with the C library's exp/log
// (src/vx27_deltanet.c:58-69) and its tests require the mapping to be bit-identical
// (tests/test_deltanet_exact.c:57). The C library's exp/log return the correctly
// rounded result for practically every input, so the device side computes the
// correctly rounded value as well, and the same code runs on host and device.
//
// Method (published, textbook):
//  * double-double arithmetic: Knuth's TwoSum, Dekker's FastTwoSum, and the exact
//    product via fused multiply-add (a*b = p + fma(a, b, -p));
//  * exp: Cody-Waite style reduction x = k ln2 + r with ln2 held as three doubles,
//    r scaled by 2^-8, Taylor series of degree 11 in double-double (Horner), then 8
//    squarings: e^x = 2^k (e^{r/256})^256. Relative error of the double-double result
//    is about 2^-92, so the final rounding is wrong only when e^x lies within ~2^-92
//    relative of a rounding boundary;
//  * log: one Newton step on exp starting from the platform log (any starting value
//    within a few ulps works): log y = l0 + log1p(y e^-l0 - 1), with the correction
//    computed in double-double.
// Results in the subnormal range (x < -708.39 for exp) may be double-rounded.
// Constants: ln2 split and 1/n! as double-double pairs, produced by tests/gen_ddconst.py.
//
// Every operation goes through the macros below so that no compiler contraction into
// FMA changes rounding between the host and the device builds.
#pragma once
#include <math.h>

#if defined(__CUDACC__)
#define VX_HD __host__ __device__ __forceinline__
#else
#define VX_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define DD_ADD(a, b) __dadd_rn((a), (b))
#define DD_SUB(a, b) __dsub_rn((a), (b))
#define DD_MUL(a, b) __dmul_rn((a), (b))
#define DD_FMA(a, b, c) __fma_rn((a), (b), (c))
#define DD_DIV(a, b) __ddiv_rn((a), (b))
#else
#define DD_ADD(a, b) ((double)(a) + (double)(b))
#define DD_SUB(a, b) ((double)(a) - (double)(b))
#define DD_MUL(a, b) ((double)(a) * (double)(b))
#define DD_FMA(a, b, c) fma((a), (b), (c))
#define DD_DIV(a, b) ((double)(a) / (double)(b))
#endif

typedef struct { double hi, lo; } vx_dd;

VX_HD vx_dd vx_two_sum(double a, double b) {
    double s = DD_ADD(a, b);
    double bb = DD_SUB(s, a);
    double e = DD_ADD(DD_SUB(a, DD_SUB(s, bb)), DD_SUB(b, bb));
    vx_dd r = {s, e};
    return r;
}
VX_HD vx_dd vx_fast_two_sum(double a, double b) { /* requires |a| >= |b| or a == 0 */
    double s = DD_ADD(a, b);
    double e = DD_SUB(b, DD_SUB(s, a));
    vx_dd r = {s, e};
    return r;
}
VX_HD vx_dd vx_two_prod(double a, double b) {
    double p = DD_MUL(a, b);
    double e = DD_FMA(a, b, -p);
    vx_dd r = {p, e};
    return r;
}
VX_HD vx_dd vx_dd_add(vx_dd a, vx_dd b) {
    vx_dd s = vx_two_sum(a.hi, b.hi);
    vx_dd t = vx_two_sum(a.lo, b.lo);
    s.lo = DD_ADD(s.lo, t.hi);
    s = vx_fast_two_sum(s.hi, s.lo);
    s.lo = DD_ADD(s.lo, t.lo);
    return vx_fast_two_sum(s.hi, s.lo);
}
VX_HD vx_dd vx_dd_mul(vx_dd a, vx_dd b) {
    vx_dd p = vx_two_prod(a.hi, b.hi);
    double cross = DD_ADD(DD_MUL(a.hi, b.lo), DD_MUL(a.lo, b.hi));
    p.lo = DD_ADD(p.lo, cross);
    return vx_fast_two_sum(p.hi, p.lo);
}
VX_HD vx_dd vx_dd_mul_d(vx_dd a, double b) {
    vx_dd p = vx_two_prod(a.hi, b);
    p.lo = DD_ADD(p.lo, DD_MUL(a.lo, b));
    return vx_fast_two_sum(p.hi, p.lo);
}

/* 1/n!, n = 0..11, as (hi, lo) */
#define VX_INV_FACT_HI(n) ( \
    (n) == 0 ? 0x1.0p+0 : (n) == 1 ? 0x1.0p+0 : (n) == 2 ? 0x1.0p-1 : \
    (n) == 3 ? 0x1.5555555555555p-3 : (n) == 4 ? 0x1.5555555555555p-5 : \
    (n) == 5 ? 0x1.1111111111111p-7 : (n) == 6 ? 0x1.6c16c16c16c17p-10 : \
    (n) == 7 ? 0x1.a01a01a01a01ap-13 : (n) == 8 ? 0x1.a01a01a01a01ap-16 : \
    (n) == 9 ? 0x1.71de3a556c734p-19 : (n) == 10 ? 0x1.27e4fb7789f5cp-22 : \
    0x1.ae64567f544e4p-26)
#define VX_INV_FACT_LO(n) ( \
    (n) <= 2 ? 0.0 : (n) == 3 ? 0x1.5555555555555p-57 : (n) == 4 ? 0x1.5555555555555p-59 : \
    (n) == 5 ? 0x1.1111111111111p-63 : (n) == 6 ? -0x1.f49f49f49f49fp-65 : \
    (n) == 7 ? 0x1.a01a01a01a01ap-73 : (n) == 8 ? 0x1.a01a01a01a01ap-76 : \
    (n) == 9 ? -0x1.c154f8ddc6c00p-73 : (n) == 10 ? 0x1.cbbc05b4fa99ap-76 : \
    -0x1.c062e06d1f209p-80)

#define VX_LN2_1 0x1.62e42fefa39efp-1
#define VX_LN2_2 0x1.abc9e3b39803fp-56
#define VX_LN2_3 0x1.7b57a079a1934p-111
#define VX_LOG2E 0x1.71547652b82fep+0

/* e^x = (hi + lo) * 2^k for |x| <= 745.2; caller handles the extremes. */
VX_HD vx_dd vx_exp_dd(double x, int *k_out) {
    double kd = rint(DD_MUL(x, VX_LOG2E));
    vx_dd p1 = vx_two_prod(kd, VX_LN2_1);
    vx_dd r = vx_two_sum(x, -p1.hi);
    vx_dd t = {-p1.lo, 0.0};
    r = vx_dd_add(r, t);
    r = vx_dd_add(r, vx_two_prod(-kd, VX_LN2_2));
    vx_dd t3 = {DD_MUL(-kd, VX_LN2_3), 0.0};
    r = vx_dd_add(r, t3);
    r.hi = DD_MUL(r.hi, 0x1.0p-8);
    r.lo = DD_MUL(r.lo, 0x1.0p-8);
    vx_dd s = {VX_INV_FACT_HI(11), VX_INV_FACT_LO(11)};
#pragma unroll
    for (int n = 10; n >= 0; n--) {
        vx_dd c = {VX_INV_FACT_HI(n), VX_INV_FACT_LO(n)};
        s = vx_dd_add(vx_dd_mul(s, r), c);
    }
#pragma unroll
    for (int i = 0; i < 8; i++) s = vx_dd_mul(s, s);
    *k_out = (int)kd;
    return s;
}

/* Correctly rounded e^x (normal range). */
VX_HD double vx_exp(double x) {
    if (x != x) return x;
    if (x > 709.782712893384) return HUGE_VAL;
    if (x < -745.2) return 0.0;
    int k;
    vx_dd s = vx_exp_dd(x, &k);
    /* 2^k may not be representable as one factor near the range ends: split it. */
    int k1 = k / 2, k2 = k - k1;
    return ldexp(ldexp(s.hi, k1), k2);
}

/* Correctly rounded log(y) for finite y > 0; other inputs follow the platform log. */
VX_HD double vx_log(double y) {
    double l0 = log(y);
    if (!(y > 0.0) || y != y || l0 == HUGE_VAL || l0 == -HUGE_VAL) return l0;
    int k;
    vx_dd e = vx_exp_dd(-l0, &k);          /* e^{-l0} = e * 2^k */
    vx_dd p = vx_dd_mul_d(e, y);           /* y e^{-l0} / 2^k */
    p.hi = ldexp(p.hi, k);
    p.lo = ldexp(p.lo, k);
    double t = DD_ADD(DD_SUB(p.hi, 1.0), p.lo);      /* y e^{-l0} - 1, |t| ~ 1e-16 */
    double corr = DD_SUB(t, DD_MUL(DD_MUL(t, t), 0.5));
    return DD_ADD(l0, corr);
}

/* The reference gate mapping (src/vx27_deltanet.c:58-69), op for op. */
VX_HD double vx_softplus(double x) {
    if (x > 20.0) return x;
    if (x < -20.0) return vx_exp(x);
    return vx_log(DD_ADD(1.0, vx_exp(x)));
}
VX_HD void vx_gate_params(double a, double A_log, double b, double dt_bias,
                          double *beta, double *g_log) {
    *beta = DD_DIV(1.0, DD_ADD(1.0, vx_exp(-b)));
    *g_log = DD_MUL(-vx_exp(A_log), vx_softplus(DD_ADD(a, dt_bias)));
}
