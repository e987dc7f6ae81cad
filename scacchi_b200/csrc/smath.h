/*
 * Deterministic float32 scalar math shared by the CUDA search kernels and by
 * the C oracle that checks them.
 *
 * Every function here uses only IEEE-754 correctly rounded operations
 * (+ - * /, sqrtf, rintf) and explicit fmaf(), so the same source produces
 * bit-identical results on the host (gcc, -ffp-contract=off) and on the GPU
 * (nvcc, -fmad=false).  That is what lets integer search decisions (argmax
 * of sampled utilities, certificate publication) agree bit-for-bit between
 * the kernels and the oracle.
 *
 * Methods (all public, none taken from a vendor math library):
 *   sm_logf    Cody-Waite reduction to m in (sqrt(1/2), sqrt(2)], then
 *              log(m) = 2 atanh(s), s = (m-1)/(m+1), Taylor series of atanh
 *              (coefficients 2/(2k+1)); ln2 split into a 16-bit head and a
 *              float tail.
 *   sm_expf    x = k ln2 + r, |r| <= ln2/2, degree-7 Taylor polynomial of
 *              e^r, exact power-of-two scaling.
 *   sm_log1pf  Goldberg/Kahan: log(u) * x / (u - 1), u = 1 + x.
 *   sm_expm1f  Kahan: (u - 1) * x / log(u), u = e^x.
 *   sm_lgammaf Stirling series (Bernoulli terms 1/12, -1/360, 1/1260) after
 *              the upward recurrence Gamma(x + 1) = x Gamma(x) to x >= 8.
 *   sm_betalnf log B(a, b): direct lgamma sum for max(a, b) < 8, otherwise
 *              the Stirling difference lgamma(b) - lgamma(a + b) written
 *              without cancellation (same split as ACM TOMS 708 "algdiv").
 *   sm_erfinvf Giles, "Approximating the erfinv function" (GPU Computing
 *              Gems Jade, 2011), single-precision coefficients as published.
 *
 * Accuracy (tests/test_oracle_pins.py: test_scalar_math_accuracy,
 * test_erfinv_tail, test_lgamma_and_betaln; against float64): log/exp/log1p <= 2 ulp,
 * lgamma/betaln absolute error <= 2e-5 * max(1, |result|), erfinv <= 4e-7
 * relative away from +-1.
 */
#ifndef SCACCHI_SMATH_H
#define SCACCHI_SMATH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define SM_FN __host__ __device__ static __forceinline__
#else
#include <math.h>
#define SM_FN static inline
#endif

SM_FN uint32_t sm_f2u(float f) {
  union { float f; uint32_t u; } v;
  v.f = f;
  return v.u;
}

SM_FN float sm_u2f(uint32_t u) {
  union { float f; uint32_t u; } v;
  v.u = u;
  return v.f;
}

#define SM_INF sm_u2f(0x7f800000u)
#define SM_NAN sm_u2f(0x7fc00000u)
/* float32 constants used by the reference through jnp.finfo(float32) */
#define SM_TINY sm_u2f(0x00800000u)      /* smallest normal, 1.17549435e-38 */
#define SM_FMIN sm_u2f(0xff7fffffu)      /* -3.40282347e38 */
#define SM_FMAX sm_u2f(0x7f7fffffu)

/* 0.693145751953125 = 45426 / 2^16 (exact in 16 bits) + float tail */
#define SM_LN2_HI 0.693145751953125f
#define SM_LN2_LO 1.42860682030941723e-06f
#define SM_INV_LN2 1.44269504088896341f

SM_FN int sm_isnan(float x) { return x != x; }
SM_FN int sm_isfinite(float x) { return (sm_f2u(x) & 0x7f800000u) != 0x7f800000u; }

SM_FN float sm_logf(float x) {
  /* Zero, negative, NaN and infinite arguments are selected at the end
   * instead of returned early, so the common path has no divergent branch;
   * positive finite arguments take exactly the operations below. */
  const int sub = sm_f2u(x) < 0x00800000u; /* subnormal (or zero): scale by 2^23 exactly */
  const float xs = sub ? x * 8388608.0f : x;
  const uint32_t u = sm_f2u(xs);
  int e = (int)((u >> 23) & 0xffu) - 127 - (sub ? 23 : 0);
  float m = sm_u2f((u & 0x007fffffu) | 0x3f800000u);
  const int big = m > 1.41421356f;
  m = big ? m * 0.5f : m;
  e += big;
  float f = m - 1.0f;
  float s = f / (2.0f + f);
  float z = s * s;
  float t = fmaf(z, 0.222222222f, 0.285714286f);  /* 2/9, 2/7 */
  t = fmaf(z, t, 0.4f);                            /* 2/5 */
  t = fmaf(z, t, 0.666666667f);                    /* 2/3 */
  float r = z * t;
  float lm = f - s * (f - r);
  float fe = (float)e;
  float v = fmaf(fe, SM_LN2_HI, fmaf(fe, SM_LN2_LO, lm));
  v = x == SM_INF ? x : v;
  return x > 0.0f ? v : (x == 0.0f ? -SM_INF : SM_NAN);
}

SM_FN float sm_ldexp_pos(float p, int k) {
  /* p * 2^k for p in [0.5, 2], k in [-151, 128]; one rounding at most */
  if (k > 127) return p * 2.0f * sm_u2f((uint32_t)(k - 1 + 127) << 23);
  if (k < -126) return (p * sm_u2f((uint32_t)(k + 64 + 127) << 23)) * 5.42101086e-20f; /* 2^-64 */
  return p * sm_u2f((uint32_t)(k + 127) << 23);
}

SM_FN float sm_expf(float x) {
  /* The special cases are selected at the end instead of returned early, so
   * the common path has no divergent branch; in-range arguments take exactly
   * the operations below. */
  float xc = x > -103.972084f ? x : -103.972084f;
  xc = xc < 88.7228394f ? xc : 88.7228394f;
  float k = rintf(xc * SM_INV_LN2);
  float r = fmaf(-k, SM_LN2_HI, xc);
  r = fmaf(-k, SM_LN2_LO, r);
  float p = fmaf(r, 1.98412698e-04f, 1.38888889e-03f);  /* 1/7!, 1/6! */
  p = fmaf(r, p, 8.33333333e-03f);                       /* 1/5! */
  p = fmaf(r, p, 4.16666667e-02f);                       /* 1/4! */
  p = fmaf(r, p, 1.66666667e-01f);                       /* 1/3! */
  p = fmaf(r, p, 0.5f);
  p = fmaf(r, p, 1.0f);
  p = fmaf(r, p, 1.0f);
  /* p * 2^k with one rounding at most (k in [-150, 128]): above 127 as
   * (p * 2^(k-1)) * 2, below -126 as (p * 2^(k+64)) * 2^-64 */
  const int ki = (int)k;
  const int kk = ki > 127 ? ki - 1 : (ki < -126 ? ki + 64 : ki);
  const float post = ki > 127 ? 2.0f : (ki < -126 ? 5.42101086e-20f : 1.0f);
  float v = (p * sm_u2f((uint32_t)(kk + 127) << 23)) * post;
  v = x > 88.7228394f ? SM_INF : v;
  v = x < -103.972084f ? 0.0f : v;
  return sm_isnan(x) ? x : v;
}

SM_FN float sm_log1pf(float x) {
  float u = 1.0f + x;
  if (u == 1.0f) return x;
  if (u == SM_INF) return SM_INF;
  if (!(u > 0.0f)) return sm_logf(u);  /* -inf at x = -1, NaN below */
  return sm_logf(u) * (x / (u - 1.0f));
}

SM_FN float sm_expm1f(float x) {
  if (sm_isnan(x)) return x;
  if (x > 88.7228394f) return SM_INF;
  if (x < -17.0f) return -1.0f;
  float u = sm_expf(x);
  if (u == 1.0f) return x;
  float um1 = u - 1.0f;
  if (um1 == -1.0f) return -1.0f;
  return um1 * (x / sm_logf(u));
}

SM_FN float sm_sqrtf(float x) { return sqrtf(x); }

/* 1/sqrt(x) with two correctly rounded operations (jax.lax.rsqrt semantics
 * up to rounding). */
SM_FN float sm_rsqrtf(float x) { return 1.0f / sqrtf(x); }

SM_FN float sm_sinhf(float t) {
  float a = t < 0.0f ? -t : t;
  float r;
  if (a < 1.0f) {
    float em1 = sm_expm1f(a);
    r = 0.5f * (em1 + em1 / (em1 + 1.0f));
  } else if (a < 88.0f) {
    float e = sm_expf(a);
    r = 0.5f * (e - 1.0f / e);
  } else {
    /* e^a / 2 without overflowing e^a */
    float e = sm_expf(0.5f * a);
    r = (0.5f * e) * e;
  }
  return t < 0.0f ? -r : r;
}

/* asinh for x >= 0 (the only use is asinh(tail_scale / min_alpha)). */
SM_FN float sm_asinhf_pos(float x) {
  if (sm_isnan(x)) return x;
  if (x > 4096.0f) return sm_logf(x) + 0.693147181f;
  float x2 = x * x;
  if (x < 0.5f) {
    /* log1p(x + x^2 / (1 + sqrt(1 + x^2))) */
    return sm_log1pf(x + x2 / (1.0f + sqrtf(1.0f + x2)));
  }
  return sm_logf(x + sqrtf(x2 + 1.0f));
}

/* jax.nn.softplus(x) = logaddexp(x, 0) = max(x, 0) + log1p(exp(-|x|)) */
SM_FN float sm_softplusf(float x) {
  if (sm_isnan(x)) return x;
  float m = x > 0.0f ? x : 0.0f;
  float a = x < 0.0f ? -x : x;
  return m + sm_log1pf(sm_expf(-a));
}

/* Stirling series tail for x >= 8: 1/(12x) - 1/(360x^3) + 1/(1260x^5) */
SM_FN float sm_stirling_tail(float x) {
  float r = 1.0f / x;
  float r2 = r * r;
  float t = fmaf(r2, 7.93650794e-04f, -2.77777778e-03f);
  t = fmaf(r2, t, 8.33333333e-02f);
  return r * t;
}

/* lgamma for x > 0 (the search only evaluates positive concentrations). */
SM_FN float sm_lgammaf(float x) {
  if (sm_isnan(x)) return x;
  if (!(x > 0.0f)) return SM_INF;
  if (x == SM_INF) return SM_INF;
  float p = 1.0f;
  float y = x;
  int shifted = 0;
  while (y < 8.0f) {
    p = p * y;
    y = y + 1.0f;
    shifted = 1;
  }
  /* 0.918938533 = log(2 pi) / 2 */
  float ly = sm_logf(y);
  float s = fmaf(y - 0.5f, ly, -y) + (0.918938533f + sm_stirling_tail(y));
  if (shifted) s = s - sm_logf(p);
  return s;
}

/* lgamma(b) - lgamma(a + b) for b >= 8, a > 0, without cancellation:
 *   a - a log b - (a + b - 1/2) log1p(a / b) + w(b) - w(a + b)
 * where w is the Stirling tail. */
SM_FN float sm_algdivf(float a, float b) {
  float l1 = sm_log1pf(a / b);
  float lb = sm_logf(b);
  float t = (a - a * lb) - ((a + b) - 0.5f) * l1;
  return t + (sm_stirling_tail(b) - sm_stirling_tail(a + b));
}

SM_FN float sm_betalnf(float a, float b) {
  float lo = a < b ? a : b;
  float hi = a < b ? b : a;
  if (hi < 8.0f) return sm_lgammaf(lo) + (sm_lgammaf(hi) - sm_lgammaf(lo + hi));
  return sm_lgammaf(lo) + sm_algdivf(lo, hi);
}

/* Giles (2011) single-precision erfinv; +-1 map to +-FLT_MAX. */
SM_FN float sm_erfinvf(float x) {
  float ax = x < 0.0f ? -x : x;
  if (ax == 1.0f) return x * SM_FMAX;
  float w = -sm_log1pf(-(x * x));
  float p;
  if (w < 5.0f) {
    w = w - 2.5f;
    p = 2.81022636e-08f;
    p = fmaf(p, w, 3.43273939e-07f);
    p = fmaf(p, w, -3.5233877e-06f);
    p = fmaf(p, w, -4.39150654e-06f);
    p = fmaf(p, w, 0.00021858087f);
    p = fmaf(p, w, -0.00125372503f);
    p = fmaf(p, w, -0.00417768164f);
    p = fmaf(p, w, 0.246640727f);
    p = fmaf(p, w, 1.50140941f);
  } else {
    w = sqrtf(w) - 3.0f;
    p = -0.000200214257f;
    p = fmaf(p, w, 0.000100950558f);
    p = fmaf(p, w, 0.00134934322f);
    p = fmaf(p, w, -0.00367342844f);
    p = fmaf(p, w, 0.00573950773f);
    p = fmaf(p, w, -0.0076224613f);
    p = fmaf(p, w, 0.00943887047f);
    p = fmaf(p, w, 1.00167406f);
    p = fmaf(p, w, 2.83297682f);
  }
  return p * x;
}

#endif /* SCACCHI_SMATH_H */
