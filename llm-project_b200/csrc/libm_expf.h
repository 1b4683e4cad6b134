/* libm_expf.h - binary32 exp that returns exactly what the host C library's
 * expf() returns, usable from host C and from CUDA device code.
 *
 * Why: the reference evaluates softmax (llama.c:567) and SiLU (llama.c:585)
 * with the platform expf.  glibc's expf is not correctly rounded: on about
 * 1.7e5 binary32 inputs it returns the neighbour on the other side of a
 * rounding midpoint.  A device exp that differs in one ulp of one attention
 * weight flips int8 activation codes downstream, so bit-identical decoding needs
 * the library's exact rounding choices.
 *
 * How:
 *  1. y = exp((double)x) (accurate to about 1 ulp of double, i.e. 2^-29 of a
 *     float ulp), f = y rounded to float.
 *  2. Let m be the rounding midpoint next to y and d = |y - m| in float ulps.
 *     If d > LX_WINDOW the host libm rounds correctly there (its misroundings all
 *     lie within 0.0017 ulp of a midpoint; the generator checks this bound on
 *     every input) and f is returned.
 *  3. Otherwise f is made correctly rounded (when d <= 2^-24 the double result
 *     cannot decide, and a double-double evaluation of exp(x) does), then the
 *     set of inputs where the host libm rounds the other way is consulted.
 *     That set is produced at build time by gen_expf_table.c, which runs this
 *     same routine against the host expf() over all 2^32 inputs.
 *
 * The double-double evaluation restates textbook methods (Dekker/Knuth error-free
 * sums and products, Cody-Waite reduction x = k ln2 + r, Taylor series of exp(r)
 * in Horner form); ln 2 is split as LX_LN2_HI + LX_LN2_LO.
 */
#ifndef LLMQ_LIBM_EXPF_H
#define LLMQ_LIBM_EXPF_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define LX_FN static __host__ __device__ __forceinline__
#else
#define LX_FN static inline
#endif

/* Inputs closer than this (in float ulps) to a rounding midpoint are checked
 * against the exception set.  The host library's misroundings all lie within
 * 0.0017 ulp of a midpoint; the generator checks every input against this
 * window less LX_MARGIN. */
#define LX_WINDOW 0x1p-9
/* exp((double)x) is within 2^-28 float ulp of exp(x), on the host and on the
 * device alike: a true distance inside LX_WINDOW - LX_MARGIN keeps y inside
 * LX_WINDOW. */
#define LX_MARGIN 0x1p-16
/* Below this the double result alone cannot decide the rounding. */
#define LX_AMBIG 0x1p-24

#define LX_LN2_HI 0x1.62e42fefa39efp-1
#define LX_LN2_LO 0x1.abc9e3b39803fp-56

LX_FN uint32_t lx_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
LX_FN float lx_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* s + e == a + b exactly */
LX_FN void lx_two_sum(double a, double b, double *s, double *e) {
  const double ss = a + b;
  const double bb = ss - a;
  *e = (a - (ss - bb)) + (b - bb);
  *s = ss;
}
/* s + e == a + b exactly when |a| >= |b| */
LX_FN void lx_fast_two_sum(double a, double b, double *s, double *e) {
  const double ss = a + b;
  *e = b - (ss - a);
  *s = ss;
}

/* exp(x) as an unevaluated sum hi + lo with relative error below 2^-95, for a
 * binary32 x with |x| <= 105 (Cody-Waite reduction, 27-term Taylor series). */
LX_FN void lx_exp_dd(double x, double *hi, double *lo) {
  const double k = rint(x * 0x1.71547652b82fep0);
  const double p1 = k * LX_LN2_HI;
  const double e1 = fma(k, LX_LN2_HI, -p1); /* p1 + e1 == k*LN2_HI */
  const double p2 = k * LX_LN2_LO;
  double s, t;
  lx_two_sum(x, -p1, &s, &t);
  t = (t - e1) - p2;
  double rh, rl;
  lx_fast_two_sum(s, t, &rh, &rl); /* r = x - k ln2, |r| <= 0.35 */
  double eh = 1.0, el = 0.0;
  for (int n = 27; n >= 1; --n) {
    /* (eh, el) <- 1 + (eh, el) * r / n */
    double ph = eh * rh;
    double pl = fma(eh, rh, -ph) + (eh * rl + el * rh);
    lx_fast_two_sum(ph, pl, &ph, &pl);
    const double qh = ph / (double)n;
    const double rem = fma(-qh, (double)n, ph);
    const double ql = (rem + pl) / (double)n;
    double sh, sl;
    lx_two_sum(1.0, qh, &sh, &sl);
    sl += ql;
    lx_fast_two_sum(sh, sl, &eh, &el);
  }
  *hi = ldexp(eh, (int)k);
  *lo = ldexp(el, (int)k);
}

/* The rounding neighbourhood of y: the two floats around it (lower < upper),
 * the midpoint between them and the float ulp there.  Returns 0 when y is a
 * float already (no rounding happened). */
LX_FN int lx_bracket(double y, float f, float *lower, float *upper, double *mid, double *ulp) {
  const double fd = (double)f;
  if (y == fd) return 0;
  if (y > fd) {
    *lower = f;
    *upper = nextafterf(f, INFINITY);
  } else {
    *upper = f;
    *lower = nextafterf(f, -INFINITY);
  }
  if (isinf(*upper)) { /* overflow boundary: FLT_MAX vs +inf */
    *mid = 0x1.ffffffp127;
    *ulp = 0x1p104;
  } else {
    *mid = 0.5 * ((double)*lower + (double)*upper);
    *ulp = (double)*upper - (double)*lower;
  }
  return 1;
}

/* Correctly rounded float exp, plus (via *near) whether it lies within
 * LX_WINDOW ulp of a midpoint, and the two candidates around that midpoint. */
LX_FN float lx_expf_cr(float x, double y, int *near, float *lower, float *upper) {
  const float f = (float)y;
  double mid = 0.0, ulp = 0.0;
  *near = 0;
  *lower = *upper = f;
  if (x != x) return x + x;
  if (!lx_bracket(y, f, lower, upper, &mid, &ulp)) return f;
  const double d = fabs(y - mid);
  if (!(d <= LX_WINDOW * ulp)) return f;
  *near = 1;
  if (d <= LX_AMBIG * ulp) {
    double h, l;
    lx_exp_dd((double)x, &h, &l);
    const double diff = (h - mid) + l;
    return diff > 0.0 ? *upper : *lower;
  }
  return f;
}

#endif /* LLMQ_LIBM_EXPF_H */
