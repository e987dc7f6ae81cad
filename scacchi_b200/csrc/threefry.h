/*
 * Threefry-2x32 (20 rounds) and the jax.random key/bit layout built on it.
 *
 * Threefry-2x32-20 is the counter-based generator of Salmon, Moraes, Dror and
 * Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC'11); rotation
 * constants {13,15,26,6} / {17,29,16,24}, key-schedule parity 0x1BD11BDA,
 * key injection after every four rounds.  Known-answer vectors from the
 * Random123 distribution are checked in tests/test_oracle_pins.py
 * (test_threefry2x32_known_answers; the split / fold_in layout below in
 * test_split_matches_documented_jax_outputs and
 * test_split_and_fold_in_counter_layout).
 *
 * The key layout follows jax.random with the partitionable threefry
 * implementation (the default of the jax version the reference pins):
 *   split(key, n)[i]     = threefry(key, (hi32(i), lo32(i)))
 *   fold_in(key, d)      = threefry(key, (0, d))
 *   random_bits(key)[i]  = x0 ^ x1 of threefry(key, (hi32(i), lo32(i)))
 * where i is the row-major flat index into the requested shape.
 * Float transforms follow jax.random.uniform / jax.random.normal:
 *   uniform01 = bitcast((bits >> 9) | 0x3f800000) - 1
 *   uniform(lo, hi) = max(lo, uniform01 * (hi - lo) + lo)
 *   normal = sqrt(2) * erfinv(uniform(nextafter(-1, 0), 1))
 */
#ifndef SCACCHI_THREEFRY_H
#define SCACCHI_THREEFRY_H

#include "smath.h"

typedef struct {
  uint32_t k0, k1;
} sk_key;

SM_FN uint32_t sk_rotl(uint32_t x, int r) {
#if defined(__CUDA_ARCH__)
  return __funnelshift_l(x, x, r);
#else
  return (x << r) | (x >> (32 - r));
#endif
}

#define SK_ROUND(r)        \
  x0 += x1;                \
  x1 = sk_rotl(x1, (r));   \
  x1 ^= x0;

SM_FN sk_key sk_threefry(sk_key key, uint32_t c0, uint32_t c1) {
  const uint32_t ks0 = key.k0, ks1 = key.k1;
  const uint32_t ks2 = ks0 ^ ks1 ^ 0x1BD11BDAu;
  uint32_t x0 = c0 + ks0;
  uint32_t x1 = c1 + ks1;
  SK_ROUND(13) SK_ROUND(15) SK_ROUND(26) SK_ROUND(6)
  x0 += ks1; x1 += ks2 + 1u;
  SK_ROUND(17) SK_ROUND(29) SK_ROUND(16) SK_ROUND(24)
  x0 += ks2; x1 += ks0 + 2u;
  SK_ROUND(13) SK_ROUND(15) SK_ROUND(26) SK_ROUND(6)
  x0 += ks0; x1 += ks1 + 3u;
  SK_ROUND(17) SK_ROUND(29) SK_ROUND(16) SK_ROUND(24)
  x0 += ks1; x1 += ks2 + 4u;
  SK_ROUND(13) SK_ROUND(15) SK_ROUND(26) SK_ROUND(6)
  x0 += ks2; x1 += ks0 + 5u;
  sk_key out;
  out.k0 = x0;
  out.k1 = x1;
  return out;
}
#undef SK_ROUND

/* jax.random.split(key, n)[i] */
SM_FN sk_key sk_split(sk_key key, uint64_t i) {
  return sk_threefry(key, (uint32_t)(i >> 32), (uint32_t)i);
}

/* jax.random.fold_in(key, d) */
SM_FN sk_key sk_fold_in(sk_key key, uint32_t d) { return sk_threefry(key, 0u, d); }

/* jax.random.bits(key, shape, uint32) at flat index i */
SM_FN uint32_t sk_bits(sk_key key, uint64_t i) {
  sk_key r = sk_threefry(key, (uint32_t)(i >> 32), (uint32_t)i);
  return r.k0 ^ r.k1;
}

SM_FN float sk_unit_from_bits(uint32_t bits) {
  return sm_u2f((bits >> 9) | 0x3f800000u) - 1.0f;
}

/* jax.random.uniform(key, shape, float32, minval=lo, maxval=hi)[i] */
SM_FN float sk_uniform(sk_key key, uint64_t i, float lo, float hi) {
  float f = sk_unit_from_bits(sk_bits(key, i));
  float v = f * (hi - lo) + lo;
  return v > lo ? v : lo;
}

/* uniform(minval=tiny, maxval=1): the draw used by the Gamma sampler and by
 * jax.random.gumbel.  (1 - tiny) rounds to 1 and f + tiny rounds to f for
 * f > 0, so this is max(tiny, f). */
SM_FN float sk_uniform_tiny(sk_key key, uint64_t i) {
  return sk_uniform(key, i, SM_TINY, 1.0f);
}

/* jax.random.normal(key, shape, float32)[i] */
SM_FN float sk_normal(sk_key key, uint64_t i) {
  /* lo = nextafter(-1, 0) = -0.99999994 */
  float u = sk_uniform(key, i, sm_u2f(0xbf7fffffu), 1.0f);
  return 1.41421354f * sm_erfinvf(u);
}

#endif /* SCACCHI_THREEFRY_H */
