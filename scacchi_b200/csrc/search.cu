// B200 kernels for the batched Dirichlet-Thompson search step.
//
// Mapping: one warp per search lane (game).  A node's action row is spread
// over the warp, action a in slot j of thread a % 32 (j = a / 32), so a row
// of the struct-of-arrays tree is read with coalesced 32-wide accesses and
// every per-node reduction (argmax, sums over actions) is a warp shuffle.
//
// Semantics follow the reference's `scacchi/dirichlet_mctx` (citations per
// function).  Floating point is bit-reproducible against the C oracle: IEEE
// operations only (built with -fmad=false), the scalar math of smath.h, and
// one canonical order for every sum over actions (per thread: slots in
// increasing order; then an xor butterfly 16, 8, 4, 2, 1).
//
// Random numbers are jax.random's threefry2x32 stream computed in-kernel at
// the counter position of each draw; because the generator is counter-based,
// the Marsaglia-Tsang proposals 1..3 are only generated when proposal 0 is
// rejected, and masked or categorical actions draw nothing.  The results are
// the same as drawing the full [4, ..., A, O] arrays.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <climits>
#include <mutex>

#include "../../include/scacchi_b200.h"
#include "synthetic_env.h"
#include "threefry.h"

namespace {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kWarpsPerBlock = 4;
constexpr int kThreads = kWarp * kWarpsPerBlock;
constexpr int kMaxHalfWidth = 512;
constexpr int8_t kNoOutcome = -1;

__device__ uint32_t g_error_flags;
std::atomic<uint64_t> g_launches{0};

// ------------------------------------------------------------------------
// tree view
// ------------------------------------------------------------------------

struct Tree {
  int B, C, A, S, E;
  int32_t *parents, *children, *to_play;
  int8_t *node_outcome;
  int32_t *node_payload;
  int8_t *edge_outcome;
  int32_t *edge_payload;
  float2 *value_prior, *value_alpha, *edge_alpha;
  uint8_t *invalid, *embedding;

  __device__ __forceinline__ size_t node(int b, int n) const { return (size_t)b * C + n; }
  __device__ __forceinline__ size_t edge(int b, int n, int a) const { return ((size_t)b * C + n) * S + a; }
  __device__ __forceinline__ bool ok(int n) const {
    if (n < 0 || n >= C) {
      atomicOr(&g_error_flags, 1u);
      return false;
    }
    return true;
  }
};

Tree make_tree(const scacchi_tree *t) {
  Tree v;
  v.B = t->batch;
  v.C = t->num_nodes;
  v.A = t->num_actions;
  v.S = t->action_stride;
  v.E = t->emb_bytes;
  v.parents = t->parents;
  v.children = t->children_index;
  v.to_play = t->node_to_play;
  v.node_outcome = t->node_outcome;
  v.node_payload = t->node_payload;
  v.edge_outcome = t->edge_outcome;
  v.edge_payload = t->edge_payload;
  v.value_prior = reinterpret_cast<float2 *>(t->node_value_prior);
  v.value_alpha = reinterpret_cast<float2 *>(t->node_value_alpha);
  v.edge_alpha = reinterpret_cast<float2 *>(t->edge_alpha);
  v.invalid = t->invalid;
  v.embedding = t->embedding;
  return v;
}

// ------------------------------------------------------------------------
// warp reductions (canonical orders shared with the oracle)
// ------------------------------------------------------------------------

__device__ __forceinline__ float butterfly_sum(float p) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) p = p + __shfl_xor_sync(kFull, p, off);
  return p;
}

template <int NS>
__device__ __forceinline__ float warp_sum(const float (&v)[NS], int A, int lane) {
  float p = 0.0f;
  bool first = true;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    if (lane + kWarp * j < A) {
      p = first ? v[j] : p + v[j];
      first = false;
    }
  }
  return butterfly_sum(p);
}

// jnp.argmax order: any NaN beats every number (first NaN wins), otherwise
// the larger value, ties to the lower index.
__device__ __forceinline__ bool beats(float av, int ai, float bv, int bi) {
  const bool an = av != av, bn = bv != bv;
  if (an || bn) return an && bn ? ai < bi : an;
  if (av != bv) return av > bv;
  return ai < bi;
}

__device__ __forceinline__ int warp_argmax(float v, int i) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float ov = __shfl_xor_sync(kFull, v, off);
    int oi = __shfl_xor_sync(kFull, i, off);
    if (beats(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
  return i;
}

__device__ __forceinline__ float warp_max_float(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float o = __shfl_xor_sync(kFull, v, off);
    v = o > v ? o : v;
  }
  return v;
}

__device__ __forceinline__ float warp_min_float(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float o = __shfl_xor_sync(kFull, v, off);
    v = o < v ? o : v;
  }
  return v;
}

__device__ __forceinline__ float2 align2(float2 v, int source, int target) {
  return source == target ? v : make_float2(v.y, v.x);
}

__device__ __forceinline__ int8_t align_cat(int8_t o, int source, int target) {
  if (o == kNoOutcome) return kNoOutcome;
  return source == target ? o : (int8_t)(1 - o);
}

// ------------------------------------------------------------------------
// Marsaglia-Tsang Dirichlet draw, action_selection.py:82-132
// ------------------------------------------------------------------------

struct DrawKeys {
  sk_key normal, accept, augment;
};

__device__ __forceinline__ DrawKeys draw_keys(sk_key key) {
  const sk_key proposal = sk_split(key, 0);
  DrawKeys k;
  k.augment = sk_split(key, 1);
  k.normal = sk_split(proposal, 0);
  k.accept = sk_split(proposal, 1);
  return k;
}

// Per-concentration constants of the Marsaglia-Tsang draw; they depend only
// on alpha, so a node's Monte Carlo population computes them once.
struct GammaShape {
  float alpha, d, c, logd;
};

__device__ __forceinline__ GammaShape gamma_shape(float alpha_in) {
  GammaShape g;
  float alpha = alpha_in > SM_TINY ? alpha_in : SM_TINY;
  if (alpha_in != alpha_in) alpha = alpha_in;
  const float shape = alpha < 1.0f ? alpha + 1.0f : alpha;
  g.alpha = alpha;
  g.d = shape - 0.333333343f;
  g.c = sm_rsqrtf(9.0f * g.d);
  g.logd = sm_logf(g.d);
  return g;
}

// log Gamma(alpha) variate at flat index idx of a [4, *shape] proposal draw
// whose proposal axis has stride `stride`.
#ifdef SCACCHI_NOINLINE_DRAW
#define SCACCHI_DRAW_INLINE __noinline__
#else
#define SCACCHI_DRAW_INLINE
#endif

// log d + log(chosen) of the draw: everything but the alpha < 1 augmentation
__device__ SCACCHI_DRAW_INLINE float log_gamma_core(const DrawKeys k, uint64_t idx, uint64_t stride,
                                                    const GammaShape g) {
  const float d = g.d, c = g.c;
  float chosen = 0.0f;
  bool found = false;
  float z0 = 0.0f;
  for (int p = 0; p < 4; ++p) {
    const uint64_t i = (uint64_t)p * stride + idx;
    const float z = sk_normal(k.normal, i);
    if (p == 0) z0 = z;
    const float base = 1.0f + c * z;
    if (!(base > 0.0f)) continue;
    const float cube = base * (base * base);
    const float u = sk_uniform_tiny(k.accept, i);
    const float z2 = z * z;
    bool accept = u < 1.0f - 0.0331f * (z2 * z2);
    if (!accept) accept = sm_logf(u) < 0.5f * z2 + d * ((1.0f - cube) + sm_logf(cube));
    if (accept) {
      chosen = cube;
      found = true;
      break;
    }
  }
  if (!found) {
    float fb = 1.0f + c * z0;
    const float floor_ = sqrtf(SM_TINY);
    fb = fb > floor_ ? fb : floor_;
    chosen = fb * (fb * fb);
  }
  return g.logd + sm_logf(chosen);
}

// the Gamma(alpha + 1) -> Gamma(alpha) augmentation, log U^(1/alpha)
__device__ __forceinline__ float gamma_augment(const DrawKeys &k, uint64_t idx, float alpha, float lg) {
  return lg + sm_logf(sk_uniform_tiny(k.augment, idx)) / alpha;
}

__device__ __forceinline__ float log_gamma_draw(const DrawKeys &k, uint64_t idx, uint64_t stride,
                                                const GammaShape &g) {
  const float lg = log_gamma_core(k, idx, stride, g);
  return g.alpha < 1.0f ? gamma_augment(k, idx, g.alpha, lg) : lg;
}

// The first proposal of the draw alone (p = 0, counter idx).  Returns true
// with v = log d + log(cube) when it is accepted, which is then exactly
// log_gamma_core's value; otherwise log_gamma_core must be run.
__device__ __forceinline__ bool gamma_first(const DrawKeys &k, uint64_t idx, float d, float c, float logd, float &v) {
  const float z = sk_normal(k.normal, idx);
  const float base = 1.0f + c * z;
  if (!(base > 0.0f)) return false;
  const float cube = base * (base * base);
  const float u = sk_uniform_tiny(k.accept, idx);
  const float z2 = z * z;
  const float lc = sm_logf(cube);
  bool accept = u < 1.0f - 0.0331f * (z2 * z2);
  if (!accept) accept = sm_logf(u) < 0.5f * z2 + d * ((1.0f - cube) + lc);
  v = logd + lc;
  return accept;
}

__device__ __forceinline__ float log_gamma_draw(const DrawKeys &k, uint64_t idx, uint64_t stride, float alpha) {
  return log_gamma_draw(k, idx, stride, gamma_shape(alpha));
}

// outcome_utility(softmax([lg0, lg1])), outcomes.py:34-35
__device__ __forceinline__ float binary_utility(float lg0, float lg1) {
  float m = lg0 > lg1 ? lg0 : lg1;
  if (lg0 != lg0 || lg1 != lg1) m = SM_NAN;
  const float e0 = sm_expf(lg0 - m), e1 = sm_expf(lg1 - m);
  const float s = e0 + e1;
  return e1 / s - e0 / s;
}

// thompson_sample (action_selection.py:135-143) for one lane of a batched
// [B, A, 2] draw; lane_base = b * A * 2, stride = B * A * 2.
template <int NS>
__device__ int warp_thompson(sk_key key, const float (&a0)[NS], const float (&a1)[NS], const bool (&masked)[NS],
                             const int8_t (&cat)[NS], bool use_cat, int A, int lane, uint64_t lane_base,
                             uint64_t stride) {
  const DrawKeys k = draw_keys(key);
  float bv = -SM_INF;
  int bi = INT_MAX;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= A) continue;
    float u;
    if (masked[j]) {
      u = -SM_INF;
    } else if (use_cat && cat[j] != kNoOutcome) {
      u = cat[j] == 1 ? 1.0f : (cat[j] == 0 ? -1.0f : 0.0f);
    } else {
      const uint64_t base = lane_base + (uint64_t)a * 2u;
      const float lg0 = log_gamma_draw(k, base, stride, a0[j]);
      const float lg1 = log_gamma_draw(k, base + 1, stride, a1[j]);
      u = binary_utility(lg0, lg1);
    }
    if (beats(u, a, bv, bi)) {
      bv = u;
      bi = a;
    }
  }
  return warp_argmax(bv, bi);
}

// posterior_best_policy (action_selection.py:146-194) for lane b of B.
template <int NS>
__device__ void warp_mc_policy(sk_key key, const float (&a0)[NS], const float (&a1)[NS], const bool (&invalid)[NS],
                               const int8_t (&cat)[NS], bool use_cat, int S, int A, int lane, int b, int B,
                               float (&policy)[NS]) {
  const uint64_t lane_base = (uint64_t)b * A * 2u, stride = (uint64_t)B * A * 2u;
  if (S == 1) {
    const int best = warp_thompson<NS>(key, a0, a1, invalid, cat, use_cat, A, lane, lane_base, stride);
#pragma unroll
    for (int j = 0; j < NS; ++j) policy[j] = (!invalid[j] && lane + kWarp * j == best) ? 1.0f : 0.0f;
    return;
  }
  const sk_key sample_key = sk_split(key, 0);
  float hits[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) hits[j] = 0.0f;
  for (int s = 0; s < S; ++s) {
    const int best =
        warp_thompson<NS>(sk_split(sample_key, (uint64_t)s), a0, a1, invalid, cat, use_cat, A, lane, lane_base, stride);
#pragma unroll
    for (int j = 0; j < NS; ++j)
      if (lane + kWarp * j == best) hits[j] = hits[j] + 1.0f;
  }
  const float fS = (float)S;
  int legal = 0;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const bool present = lane + kWarp * j < A;
    policy[j] = (present && !invalid[j]) ? hits[j] / fS : 0.0f;
    legal += present && !invalid[j];
  }
  legal = __reduce_add_sync(kFull, legal);
  const float total = warp_sum<NS>(policy, A, lane);
  const float denom = total > 1.0f ? total : 1.0f;
  const float lc = (float)(legal > 1 ? legal : 1);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    if (total > 0.0f) policy[j] = policy[j] / denom;
    else policy[j] = (invalid[j] ? 0.0f : 1.0f) / lc;
  }
}

// ------------------------------------------------------------------------
// prefix-CDF estimator, prefix_cdf.py:217-445
// ------------------------------------------------------------------------

struct PrefixScratch {
  float *lx, *l1mx, *lj, *flp, *joint;
  int *zc;
};

__device__ __forceinline__ PrefixScratch prefix_scratch(int Q) {
  extern __shared__ float smem[];
  const int w = threadIdx.x / kWarp;
  float *base = smem + (size_t)w * 6 * Q;
  PrefixScratch s;
  s.lx = base;
  s.l1mx = base + Q;
  s.lj = base + 2 * Q;
  s.flp = base + 3 * Q;
  s.joint = base + 4 * Q;
  s.zc = reinterpret_cast<int *>(base + 5 * Q);
  return s;
}

struct PrefixParams {
  int h;
  float tail, min_hr, max_hr;
};

struct PrefixLane {
  float mass, nerr, hr;
  bool finite, clipped;
  int fic;
};

__device__ __forceinline__ float log_cosh(float v) {
  const float a = v < 0.0f ? -v : v;
  return (a + sm_log1pf(sm_expf(-2.0f * a))) - sm_logf(2.0f);
}

template <int NS>
__device__ void warp_prefix_cdf(const float (&a0)[NS], const float (&a1)[NS], const bool (&invalid)[NS],
                                const int8_t (&outc)[NS], int A, int lane, const PrefixParams &P,
                                const PrefixScratch &sc, float (&policy)[NS], float (&raw)[NS], float (&dli)[NS],
                                PrefixLane &L) {
  const int h = P.h, Q = 2 * h + 1;
  bool present[NS], unres[NS], legal[NS], cwin[NS];
  int n_unres = 0;
  bool any_unres = false, any_legal = false, any_cw = false;
  float amin = SM_INF;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    present[j] = lane + kWarp * j < A;
    legal[j] = present[j] && !invalid[j];
    unres[j] = legal[j] && outc[j] == kNoOutcome;
    cwin[j] = legal[j] && outc[j] == 1;
    n_unres += unres[j];
    any_unres |= unres[j];
    any_legal |= legal[j];
    any_cw |= cwin[j];
    if (unres[j]) {
      const float v0 = a0[j] > SM_TINY ? a0[j] : SM_TINY;
      const float v1 = a1[j] > SM_TINY ? a1[j] : SM_TINY;
      if (v0 < amin) amin = v0;
      if (v1 < amin) amin = v1;
    }
  }
  n_unres = __reduce_add_sync(kFull, n_unres);
  const bool has_unres = __any_sync(kFull, any_unres);
  const bool has_legal = __any_sync(kFull, any_legal);
  const bool has_cw = __any_sync(kFull, any_cw);
  amin = warp_min_float(amin);
  // _adaptive_grid_half_range, prefix_cdf.py:68-118
  float requested = sm_asinhf_pos(P.tail / amin);
  if (!has_unres) requested = P.min_hr;
  float hr = requested;
  if (hr < P.min_hr) hr = P.min_hr;
  if (hr > P.max_hr) hr = P.max_hr;
  const bool clipped = has_unres && requested > P.max_hr;
  const float fh = (float)h;
  for (int k = lane; k < Q; k += kWarp) {
    const float unit = (float)(k - h) / fh;
    const float coord = hr * unit;
    const float logit = sm_sinhf(coord);
    sc.lx[k] = -sm_softplusf(-logit);
    sc.l1mx[k] = -sm_softplusf(logit);
    sc.lj[k] = log_cosh(coord);
  }
  __syncwarp();
  const float hstep = 0.5f * (hr / fh);
  // per-action Beta log-density normalisation
  float w[NS], l[NS], bl[NS], scale[NS], safe[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    w[j] = unres[j] ? (a1[j] > SM_TINY ? a1[j] : SM_TINY) : 1.0f;
    l[j] = unres[j] ? (a0[j] > SM_TINY ? a0[j] : SM_TINY) : 1.0f;
    bl[j] = sm_betalnf(w[j], l[j]);
    float s = -SM_INF;
    bool nan = false;
    for (int k = 0; k < Q; ++k) {
      const float ld = ((w[j] * sc.lx[k] + l[j] * sc.l1mx[k]) - bl[j]) + sc.lj[k];
      nan |= ld != ld;
      if (ld > s) s = ld;
    }
    scale[j] = nan ? SM_NAN : s;
    float run = 0.0f, prev = 0.0f;
    for (int k = 0; k < Q; ++k) {
      const float ld = ((w[j] * sc.lx[k] + l[j] * sc.l1mx[k]) - bl[j]) + sc.lj[k];
      const float d = unres[j] ? sm_expf(ld - scale[j]) : 0.0f;
      if (k > 0) run = run + hstep * (prev + d);
      prev = d;
    }
    dli[j] = unres[j] ? scale[j] + sm_logf(run) : 0.0f;
    safe[j] = run > 0.0f ? run : 1.0f;
  }
  // per grid point: leave-one-out log products and the joint maximum CDF
  {
    float run[NS], prev[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) run[j] = prev[j] = 0.0f;
    for (int k = 0; k < Q; ++k) {
      float flc[NS], lj[NS];
      int zero = 0;
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        const float ld = ((w[j] * sc.lx[k] + l[j] * sc.l1mx[k]) - bl[j]) + sc.lj[k];
        const float d = unres[j] ? sm_expf(ld - scale[j]) : 0.0f;
        if (k > 0) run[j] = run[j] + hstep * (prev[j] + d);
        prev[j] = d;
        const float c = run[j] / safe[j];
        const bool pos = c > 0.0f;
        const float f = pos ? sm_logf(c) : 0.0f;
        zero += present[j] && unres[j] && !pos;
        flc[j] = unres[j] ? f : 0.0f;
        const float m = f < 0.0f ? f : 0.0f;
        lj[j] = unres[j] ? (pos ? m : -SM_INF) : 0.0f;
      }
      zero = __reduce_add_sync(kFull, zero);
      const float flp = warp_sum<NS>(flc, A, lane);
      const float lsum = warp_sum<NS>(lj, A, lane);
      if (lane == 0) {
        sc.zc[k] = zero;
        sc.flp[k] = flp;
        sc.joint[k] = sm_expf(lsum);
      }
    }
  }
  __syncwarp();
  // _maximum_cdf endpoint pins and running maximum, prefix_cdf.py:186-214
  if (lane == 0) {
    sc.joint[0] = has_unres ? 0.0f : 1.0f;
    sc.joint[Q - 1] = 1.0f;
    for (int k = 1; k < Q; ++k) {
      const float p = sc.joint[k - 1], c = sc.joint[k];
      if (p != p || (c == c && p > c)) sc.joint[k] = p;
    }
    sc.joint[Q - 1] = 1.0f;
  }
  __syncwarp();
  // allocation of joint increments in proportion to winner contributions
  float prob[NS];
  int fic = 0;
  {
    float run[NS], prev[NS], prev_int[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) run[j] = prev[j] = prev_int[j] = prob[j] = 0.0f;
    const float uden = (float)(n_unres > 1 ? n_unres : 1);
    for (int k = 0; k < Q; ++k) {
      float contrib[NS];
      const int zc = sc.zc[k];
      const float flp = sc.flp[k];
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        const float ld = ((w[j] * sc.lx[k] + l[j] * sc.l1mx[k]) - bl[j]) + sc.lj[k];
        const float d = unres[j] ? sm_expf(ld - scale[j]) : 0.0f;
        if (k > 0) run[j] = run[j] + hstep * (prev[j] + d);
        prev[j] = d;
        const float c = run[j] / safe[j];
        const bool pos = c > 0.0f;
        const float f = pos ? sm_logf(c) : 0.0f;
        const int zf = unres[j] && !pos;
        const float olp = (zc - zf) > 0 ? -SM_INF : flp - f;
        const float integ = (d / safe[j]) * sm_expf(olp);
        if (k > 0) {
          const float cc = hstep * (prev_int[j] + integ);
          contrib[j] = cc > 0.0f ? cc : (cc != cc ? cc : 0.0f);
        } else {
          contrib[j] = 0.0f;
        }
        prev_int[j] = integ;
      }
      if (k == 0) continue;
      const float score = warp_sum<NS>(contrib, A, lane);
      float jinc = sc.joint[k] - sc.joint[k - 1];
      jinc = jinc > 0.0f ? jinc : (jinc != jinc ? jinc : 0.0f);
      const bool sp = score > 0.0f;
      fic += (!sp && jinc > 0.0f) ? 1 : 0;
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        const float wgt = sp ? contrib[j] / score : (unres[j] ? 1.0f : 0.0f) / uden;
        prob[j] = prob[j] + wgt * jinc;
      }
    }
  }
  // _finalize_policy, prefix_cdf.py:121-183
  int first_cw = INT_MAX;
  float cv = -SM_INF;
  int ci = INT_MAX;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (!present[j]) continue;
    if (cwin[j] && a < first_cw) first_cw = a;
    const float s = legal[j] ? (float)outc[j] : -SM_INF;
    if (beats(s, a, cv, ci)) {
      cv = s;
      ci = a;
    }
  }
  first_cw = __reduce_min_sync(kFull, first_cw);
  const int cbest = has_cw ? first_cw : warp_argmax(cv, ci);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const float r = (has_cw || !has_unres) ? (a == cbest ? 1.0f : 0.0f) : (unres[j] ? prob[j] : 0.0f);
    raw[j] = legal[j] ? r : 0.0f;
  }
  const float mass = warp_sum<NS>(raw, A, lane);
  const float nerr = fabsf(mass - (has_legal ? 1.0f : 0.0f));
  const float smass = mass > 0.0f ? mass : 1.0f;
  bool fin = true;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    float p = raw[j] / smass;
    p = has_legal ? p : 0.0f;
    policy[j] = p;
    if (present[j]) {
      fin = fin && sm_isfinite(p) && sm_isfinite(raw[j]);
      if (unres[j] && !sm_isfinite(dli[j])) fin = false;
    }
  }
  fin = __all_sync(kFull, fin) && sm_isfinite(mass) && sm_isfinite(nerr) && sm_isfinite(hr);
  L.mass = mass;
  L.nerr = nerr;
  L.hr = hr;
  L.finite = fin;
  L.clipped = clipped;
  L.fic = fic;
  __syncwarp();
}

// ------------------------------------------------------------------------
// posterior repair, posterior_updates.py:40-367
// ------------------------------------------------------------------------

struct UpdateParams {
  int rule, kappa_ge_one, samples;
  float inv_kappa, kappa, density_tol;
  PrefixParams prefix;
};

UpdateParams make_params(const scacchi_update_params *p) {
  UpdateParams u;
  u.rule = p->rule;
  u.kappa_ge_one = p->kappa_ge_one;
  u.samples = p->samples;
  u.inv_kappa = p->inv_kappa;
  u.kappa = p->kappa;
  u.density_tol = p->density_tol;
  u.prefix.h = p->half_width;
  u.prefix.tail = p->tail_scale;
  u.prefix.min_hr = p->min_half_range;
  u.prefix.max_hr = p->max_half_range;
  return u;
}

template <int NS>
struct NodeCtx {
  bool active, leaf_active;
  int leaf_action, leaf_to_play, node_to_play, node_payload;
  float2 leaf_value, value_prior, value_alpha;
  float ea0[NS], ea1[NS];
  int ep[NS];
  int8_t eo[NS];
  bool inv[NS];
  bool cvis[NS];
  float2 cprior[NS], cvalue[NS];
  int cpay[NS];
  int8_t cout[NS];
  int ctp[NS];
};

template <int NS>
struct NodeUpdate {
  float ea0[NS], ea1[NS];
  int ep[NS];
  float2 value_alpha;
  int n_down;
  bool unsafe;
};

// _repair_inputs + rule + _repair_from_policy for one lane (b of B).
template <int NS>
__device__ void warp_posterior_update(sk_key update_key, const NodeCtx<NS> &c, int A, int lane,
                                      const UpdateParams &P, const PrefixScratch &sc, int b, int B,
                                      NodeUpdate<NS> &out) {
  float eff0[NS], eff1[NS], cache0[NS], cache1[NS];
  int delta = 0;
  const int leaf_action = c.leaf_action < 0 ? c.leaf_action + A : c.leaf_action;
  const float2 direct = align2(c.leaf_value, c.leaf_to_play, c.node_to_play);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const bool present = a < A;
    const bool unresolved = c.eo[j] == kNoOutcome;
    float e0 = c.ea0[j], e1 = c.ea1[j];
    int ep = c.ep[j];
    if (c.leaf_active && a == leaf_action && unresolved) {
      e0 = direct.x;
      e1 = direct.y;
      ep = ep + 1;
    }
    if (c.active && c.cvis[j] && c.cout[j] == kNoOutcome && c.cpay[j] > 0 && unresolved) {
      const float2 cv = align2(c.cvalue[j], c.ctp[j], c.node_to_play);
      e0 = cv.x;
      e1 = cv.y;
      ep = 1 + c.cpay[j];
    }
    out.ea0[j] = e0;
    out.ea1[j] = e1;
    out.ep[j] = ep;
    if (c.cvis[j] && unresolved && ep <= 0) {
      const float2 cp = align2(c.cprior[j], c.ctp[j], c.node_to_play);
      eff0[j] = cp.x;
      eff1[j] = cp.y;
    } else {
      eff0[j] = e0;
      eff1[j] = e1;
    }
    if (!unresolved) {
      const float s = eff0[j] + eff1[j];
      cache0[j] = s * (c.eo[j] == 0 ? 1.0f : 0.0f);
      cache1[j] = s * (c.eo[j] == 1 ? 1.0f : 0.0f);
    } else {
      cache0[j] = eff0[j];
      cache1[j] = eff1[j];
    }
    if (present && unresolved && !c.inv[j]) delta += ep - c.ep[j];
  }
  delta = __reduce_add_sync(kFull, delta);
  const int n_down = c.node_payload + delta;
  float policy[NS];
  bool unsafe = false;
  if (P.rule == 1) {
    float raw[NS], dli[NS];
    PrefixLane L;
    warp_prefix_cdf<NS>(eff0, eff1, c.inv, c.eo, A, lane, P.prefix, sc, policy, raw, dli, L);
    float derr = 0.0f;
    bool dnan = false;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      if (lane + kWarp * j >= A) continue;
      const float v = fabsf(dli[j]);
      dnan |= v != v;
      if (v > derr) derr = v;
    }
    derr = warp_max_float(derr);
    dnan = __any_sync(kFull, dnan);
    const bool too_large = !dnan && derr > P.density_tol;
    unsafe = c.active && (L.clipped || !L.finite || too_large);
    if (unsafe) warp_mc_policy<NS>(update_key, eff0, eff1, c.inv, c.eo, true, P.samples, A, lane, b, B, policy);
  } else {
    warp_mc_policy<NS>(update_key, eff0, eff1, c.inv, c.eo, true, P.samples, A, lane, b, B, policy);
  }
  // mix_value_prior, posterior_updates.py:40-63
  float t0[NS], t1[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    t0[j] = policy[j] * cache0[j];
    t1[j] = policy[j] * cache1[j];
  }
  const float w0 = warp_sum<NS>(t0, A, lane), w1 = warp_sum<NS>(t1, A, lane);
  const float n = (float)n_down;
  float pw, dw;
  if (P.kappa_ge_one) {
    const float rc = n * P.inv_kappa;
    const float den = 1.0f + rc;
    pw = 1.0f / den;
    dw = rc / den;
  } else {
    const float den = P.kappa + n;
    pw = P.kappa / den;
    dw = n / den;
  }
  const float2 repaired = make_float2(pw * c.value_prior.x + dw * w0, pw * c.value_prior.y + dw * w1);
  out.value_alpha = (c.active && n_down > 0) ? repaired : c.value_alpha;
  out.n_down = n_down;
  out.unsafe = unsafe;
}

// gather a node context (utils.py:35-50)
template <int NS>
__device__ void gather_ctx(const Tree &T, int b, int n, int lane, NodeCtx<NS> &c) {
  const size_t ni = T.node(b, n);
  c.node_to_play = T.to_play[ni];
  c.node_payload = T.node_payload[ni];
  c.value_prior = T.value_prior[ni];
  c.value_alpha = T.value_alpha[ni];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= T.A) {
      c.ea0[j] = c.ea1[j] = 1.0f;
      c.ep[j] = 0;
      c.eo[j] = kNoOutcome;
      c.inv[j] = true;
      c.cvis[j] = false;
      c.cprior[j] = c.cvalue[j] = make_float2(1.0f, 1.0f);
      c.cpay[j] = 0;
      c.cout[j] = kNoOutcome;
      c.ctp[j] = 0;
      continue;
    }
    const size_t e = T.edge(b, n, a);
    const float2 ea = T.edge_alpha[e];
    c.ea0[j] = ea.x;
    c.ea1[j] = ea.y;
    c.ep[j] = T.edge_payload[e];
    c.eo[j] = T.edge_outcome[e];
    c.inv[j] = T.invalid[e] != 0;
    int child = T.children[e];
    c.cvis[j] = child != -1;
    if (child != -1 && !T.ok(child)) child = -1;
    const size_t ci = T.node(b, child != -1 ? child : 0);
    c.cprior[j] = T.value_prior[ci];
    c.cvalue[j] = T.value_alpha[ci];
    c.cpay[j] = T.node_payload[ci];
    c.cout[j] = T.node_outcome[ci];
    c.ctp[j] = T.to_play[ci];
  }
}

// _set_node_update (utils.py:53-64) and _categorize_node_and_publish
// (utils.py:67-124, binary outcomes) for an active lane.
template <int NS>
__device__ void store_and_publish(const Tree &T, int b, int n, int lane, const NodeCtx<NS> &c,
                                  const NodeUpdate<NS> &u) {
  const size_t ni = T.node(b, n);
  bool any_legal = false, any_open = false, any_win = false;
  int shortest_win = INT_MAX, longest_loss = INT_MIN;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= T.A) continue;
    const size_t e = T.edge(b, n, a);
    if (c.eo[j] == kNoOutcome) {
      T.edge_payload[e] = u.ep[j];
      T.edge_alpha[e] = make_float2(u.ea0[j], u.ea1[j]);
    }
    const bool legal = !c.inv[j];
    const bool known = legal && c.eo[j] != kNoOutcome;
    any_legal |= legal;
    any_open |= legal && !known;
    if (known && c.eo[j] == 1) {
      any_win = true;
      if (c.ep[j] < shortest_win) shortest_win = c.ep[j];
    }
    if (known && c.eo[j] == 0 && c.ep[j] > longest_loss) longest_loss = c.ep[j];
  }
  const bool has_legal = __any_sync(kFull, any_legal);
  const bool all_cat = has_legal && !__any_sync(kFull, any_open);
  const bool has_win = __any_sync(kFull, any_win);
  shortest_win = __reduce_min_sync(kFull, shortest_win);
  longest_loss = __reduce_max_sync(kFull, longest_loss);
  if (lane == 0) {
    T.node_payload[ni] = u.n_down;
    T.value_alpha[ni] = u.value_alpha;
  }
  const int8_t candidate = has_win ? 1 : (all_cat ? 0 : kNoOutcome);
  const int cdist = has_win ? shortest_win : longest_loss;
  const int8_t old_outcome = T.node_outcome[ni];
  const bool publish_node = old_outcome == kNoOutcome && candidate != kNoOutcome;
  if (publish_node) {
    int parent = T.parents[ni];
    const bool has_parent = parent != -1 && T.ok(parent);
    const int sp = has_parent ? parent : 0;
    int first = INT_MAX;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int a = lane + kWarp * j;
      if (a < T.A && T.children[T.edge(b, sp, a)] == n && a < first) first = a;
    }
    first = __reduce_min_sync(kFull, first);
    const bool has_incoming = first != INT_MAX;
    const int ia = has_incoming ? first : 0;
    if (lane == 0) {
      const size_t pe = T.edge(b, sp, ia), pn = T.node(b, sp);
      const bool publish_edge = has_parent && has_incoming && T.edge_outcome[pe] == kNoOutcome;
      const int new_support = T.node_payload[pn] + 1 + u.n_down - T.edge_payload[pe];
      const int8_t aligned = align_cat(candidate, T.to_play[ni], T.to_play[pn]);
      if (publish_edge) T.node_payload[pn] = new_support;
      T.node_payload[ni] = cdist;
      T.node_outcome[ni] = candidate;
      if (publish_edge) {
        T.edge_outcome[pe] = aligned;
        T.edge_payload[pe] = cdist + 1;
      }
    }
  }
  __syncwarp();
}

#include "lane_cta.cuh"

// ------------------------------------------------------------------------
// kernels
// ------------------------------------------------------------------------

__device__ __forceinline__ int warp_lane_index() {
  return (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) / kWarp);
}

// instantiate_tree_from_root, tree.py:245-277
__global__ void tree_init_kernel(Tree T, const float2 *root_value, const float2 *root_av, const uint8_t *root_inv,
                                 const int8_t *root_term, const int32_t *root_tp, const uint8_t *root_emb,
                                 int full) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= T.B) return;
  const int last = full ? T.C : 1;
  for (int n = 0; n < last; ++n) {
    const bool root = n == 0;
    const size_t ni = T.node(b, n);
    for (int a = lane; a < T.A; a += kWarp) {
      const size_t e = T.edge(b, n, a);
      T.children[e] = -1;
      T.edge_outcome[e] = kNoOutcome;
      T.edge_payload[e] = 0;
      T.invalid[e] = root ? root_inv[(size_t)b * T.A + a] : 1;
      T.edge_alpha[e] = root ? root_av[(size_t)b * T.A + a] : make_float2(1.0f, 1.0f);
    }
    for (int i = lane; i < T.E; i += kWarp)
      T.embedding[ni * T.E + i] = (root && root_emb) ? root_emb[(size_t)b * T.E + i] : 0;
    if (lane == 0) {
      T.parents[ni] = -1;
      T.to_play[ni] = root ? root_tp[b] : 0;
      T.node_outcome[ni] = root ? root_term[b] : kNoOutcome;
      T.node_payload[ni] = 0;
      const float2 v = root ? root_value[b] : make_float2(1.0f, 1.0f);
      T.value_prior[ni] = v;
      T.value_alpha[ni] = v;
    }
  }
}

template <int NS>
__device__ bool warp_any_searchable(const Tree &T, int b, int n, int lane) {
  bool s = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a < T.A) {
      const size_t e = T.edge(b, n, a);
      s |= !T.invalid[e] && T.edge_outcome[e] == kNoOutcome;
    }
  }
  return __any_sync(kFull, s);
}

// simulate / _simulate_one, search.py:21-78
template <int NS>
__global__ void __launch_bounds__(kThreads) simulate_kernel(Tree T, const uint32_t *key, int max_depth,
                                                            int32_t *out_parent, int32_t *out_action,
                                                            uint8_t *out_active, uint8_t *parent_emb,
                                                            unsigned long long *stats) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= T.B) return;
  const sk_key sim_key = {key[0], key[1]};
  sk_key k = sk_split(sim_key, (uint64_t)b);
  const bool root_active = T.node_outcome[T.node(b, 0)] == kNoOutcome && warp_any_searchable<NS>(T, b, 0, lane);
  int node = 0, next = 0, action = 0, depth = 0;
  bool cont = root_active;
  const uint64_t stride = (uint64_t)T.A * 2u;
  unsigned long long visited_nodes = 0, prior_gathers = 0;
  while (cont) {
    visited_nodes += 1;
    const sk_key next_key = sk_split(k, 0), sel_key = sk_split(k, 1);
    node = next;
    const int player = T.to_play[T.node(b, node)];
    float a0[NS], a1[NS];
    bool masked[NS];
    int8_t cat[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int a = lane + kWarp * j;
      cat[j] = kNoOutcome;
      masked[j] = true;
      a0[j] = a1[j] = 1.0f;
      if (a >= T.A) continue;
      const size_t e = T.edge(b, node, a);
      masked[j] = T.invalid[e] || T.edge_outcome[e] != kNoOutcome;
      if (masked[j]) continue;
      const int child = T.children[e];
      float2 alpha;
      if (child != -1 && T.edge_payload[e] <= 0 && T.ok(child)) {
        const size_t ci = T.node(b, child);
        alpha = align2(T.value_prior[ci], T.to_play[ci], player);
        prior_gathers += 1;
      } else {
        alpha = T.edge_alpha[e];
      }
      a0[j] = alpha.x;
      a1[j] = alpha.y;
    }
    action = warp_thompson<NS>(sel_key, a0, a1, masked, cat, false, T.A, lane, 0, stride);
    int child = T.children[T.edge(b, node, action)];
    if (child != -1 && !T.ok(child)) child = -1;
    const bool visited = child != -1;
    const int safe = visited ? child : 0;
    depth += 1;
    const bool selectable =
        T.node_outcome[T.node(b, safe)] == kNoOutcome && warp_any_searchable<NS>(T, b, safe, lane);
    cont = visited && selectable && depth < max_depth;
    next = child;
    k = next_key;
  }
  if (lane == 0) {
    out_parent[b] = node;
    out_action[b] = action;
    out_active[b] = root_active;
  }
  if (stats) {
    prior_gathers = __reduce_add_sync(kFull, (unsigned)prior_gathers);
    if (lane == 0) {
      atomicAdd(stats + 0, visited_nodes);
      atomicAdd(stats + 1, prior_gathers);
    }
  }
  if (parent_emb) {
    const int p = root_active ? node : 0;
    const uint8_t *src = T.embedding + T.node(b, p) * T.E;
    for (int i = lane; i < T.E; i += kWarp) parent_emb[(size_t)b * T.E + i] = src[i];
  }
}

// expand + _set_expanded_node, search.py:81-143
__global__ void __launch_bounds__(kThreads) expand_kernel(Tree T, int new_node, const int32_t *sim_parent,
                                                          const int32_t *sim_action, const uint8_t *sim_active,
                                                          const float2 *step_value, const float2 *step_av,
                                                          const uint8_t *step_inv, const int8_t *step_term,
                                                          const int32_t *step_tp, const uint8_t *child_emb,
                                                          int lazy) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= T.B) return;
  const bool active = sim_active[b] != 0;
  int parent = active ? sim_parent[b] : 0;
  int action = active ? sim_action[b] : 0;
  if (!T.ok(parent) || action < 0 || action >= T.A) {
    if (lane == 0) atomicOr(&g_error_flags, 1u);
    return;
  }
  const size_t pe = T.edge(b, parent, action), pn = T.node(b, parent);
  const int child = T.children[pe];
  const bool init = active && child == -1;
  const int8_t outcome = step_term[b];
  const int8_t aligned = align_cat(outcome, step_tp[b], T.to_play[pn]);
  const bool publish = active && outcome != kNoOutcome;
  const int parent_support = T.node_payload[pn] + (1 - T.edge_payload[pe]);
  __syncwarp();
  if (new_node >= 1 && new_node < T.C && (init || lazy)) {
    const size_t ni = T.node(b, new_node);
    for (int a = lane; a < T.A; a += kWarp) {
      const size_t e = T.edge(b, new_node, a);
      T.invalid[e] = init ? step_inv[(size_t)b * T.A + a] : 1;
      T.edge_alpha[e] = init ? step_av[(size_t)b * T.A + a] : make_float2(1.0f, 1.0f);
      if (lazy) {
        T.children[e] = -1;
        T.edge_outcome[e] = kNoOutcome;
        T.edge_payload[e] = 0;
      }
    }
    for (int i = lane; i < T.E; i += kWarp)
      T.embedding[ni * T.E + i] = (init && child_emb) ? child_emb[(size_t)b * T.E + i] : 0;
    if (lane == 0) {
      if (init) {
        T.parents[ni] = parent;
        T.to_play[ni] = step_tp[b];
        T.node_outcome[ni] = outcome;
        T.value_prior[ni] = step_value[b];
        T.value_alpha[ni] = step_value[b];
        T.children[pe] = new_node;
      } else {
        T.parents[ni] = -1;
        T.to_play[ni] = 0;
        T.node_outcome[ni] = kNoOutcome;
        T.value_prior[ni] = make_float2(1.0f, 1.0f);
        T.value_alpha[ni] = make_float2(1.0f, 1.0f);
      }
      if (lazy) T.node_payload[ni] = 0;
    }
  }
  if (lane == 0 && publish) {
    T.node_payload[pn] = parent_support;
    T.edge_outcome[pe] = aligned;
    T.edge_payload[pe] = 1;
  }
}

// backward, search.py:146-171
template <int NS>
__global__ void __launch_bounds__(kThreads) backward_kernel(Tree T, const uint32_t *key, const int32_t *sim_parent,
                                                            const int32_t *sim_action, const uint8_t *sim_active,
                                                            const float2 *step_value, const int32_t *step_tp,
                                                            UpdateParams P, unsigned long long *stats) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  const PrefixScratch sc = prefix_scratch(2 * P.prefix.h + 1);
  if (b >= T.B) return;
  bool active = sim_active[b] != 0;
  int node = active ? sim_parent[b] : 0;
  if (!T.ok(node)) return;
  bool leaf_active = active;
  sk_key k = {key[0], key[1]};
  NodeCtx<NS> c;
  NodeUpdate<NS> u;
  c.leaf_action = sim_action[b];
  c.leaf_value = step_value[b];
  c.leaf_to_play = step_tp[b];
  unsigned long long unsafe = 0, nodes = 0, child_gathers = 0;
  for (int level = 0; active && level < T.C; ++level) {
    const sk_key next_key = sk_split(k, 0), update_key = sk_split(k, 1);
    c.active = true;
    c.leaf_active = leaf_active;
    gather_ctx<NS>(T, b, node, lane, c);
    warp_posterior_update<NS>(update_key, c, T.A, lane, P, sc, b, T.B, u);
    unsafe += u.unsafe;
    nodes += 1;
    if (stats) {
      int cv = 0;
#pragma unroll
      for (int j = 0; j < NS; ++j) cv += c.cvis[j] && lane + kWarp * j < T.A;
      child_gathers += __reduce_add_sync(kFull, cv);
    }
    store_and_publish<NS>(T, b, node, lane, c, u);
    const bool up = node != 0;
    int parent = T.parents[T.node(b, node)];
    if (up && !T.ok(parent)) break;
    node = up ? parent : 0;
    active = up;
    leaf_active = false;
    k = next_key;
  }
  if (stats && lane == 0) {
    atomicAdd(stats + 0, nodes);
    atomicAdd(stats + 1, child_gathers);
    if (unsafe) atomicAdd(stats + 2, unsafe);
  }
}

// root policy, policies.py:28-42
template <int NS>
__global__ void __launch_bounds__(kThreads) root_policy_kernel(Tree T, const uint32_t *key, const uint8_t *invalid,
                                                               int samples, float *weights, int32_t *action) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= T.B) return;
  const sk_key policy_key = {key[0], key[1]};
  const int A = T.A;
  const size_t ri = T.node(b, 0);
  const int8_t root_outcome = T.node_outcome[ri];
  float w[NS];
  bool inv[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    inv[j] = a < A ? invalid[(size_t)b * A + a] != 0 : true;
  }
  if (root_outcome != kNoOutcome) {
    // categorical_action: argmax(gumbel + tie logits), action_selection.py:24-59
    float score[NS];
    float best = -SM_INF;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int a = lane + kWarp * j;
      score[j] = -SM_INF;
      if (a >= A) continue;
      const size_t e = T.edge(b, 0, a);
      const int8_t eo = T.edge_outcome[e];
      const float dist = (float)T.edge_payload[e];
      const bool legal = !inv[j];
      if (root_outcome == 1) score[j] = (legal && eo == 1) ? -dist : -SM_INF;
      else if (root_outcome == 0) score[j] = (legal && eo == 0) ? dist : -SM_INF;
      else score[j] = (legal && eo == 1) ? 0.0f : -SM_INF;
      if (score[j] > best) best = score[j];
    }
    best = warp_max_float(best);
    const sk_key tie_key = sk_fold_in(policy_key, 0);
    float nv = -SM_INF;
    int ni = INT_MAX, count = 0;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int a = lane + kWarp * j;
      if (a >= A) continue;
      const bool tied = sm_isfinite(score[j]) && score[j] == best;
      count += tied;
      const float g = -sm_logf(-sm_logf(sk_uniform_tiny(tie_key, (uint64_t)b * A + a)));
      const float v = g + (tied ? 0.0f : -SM_INF);
      if (beats(v, a, nv, ni)) {
        nv = v;
        ni = a;
      }
    }
    count = __reduce_add_sync(kFull, count);
    int chosen = warp_argmax(nv, ni);
    if (count == 0) chosen = 0;
#pragma unroll
    for (int j = 0; j < NS; ++j) w[j] = lane + kWarp * j == chosen ? 1.0f : 0.0f;
  } else {
    const int player = T.to_play[ri];
    float a0[NS], a1[NS];
    int8_t cat[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int a = lane + kWarp * j;
      a0[j] = a1[j] = 1.0f;
      cat[j] = kNoOutcome;
      if (a >= A) continue;
      const size_t e = T.edge(b, 0, a);
      cat[j] = T.edge_outcome[e];
      const int child = T.children[e];
      float2 alpha = T.edge_alpha[e];
      if (child != -1 && cat[j] == kNoOutcome && T.edge_payload[e] <= 0 && T.ok(child)) {
        const size_t ci = T.node(b, child);
        alpha = align2(T.value_prior[ci], T.to_play[ci], player);
      }
      a0[j] = alpha.x;
      a1[j] = alpha.y;
    }
    warp_mc_policy<NS>(policy_key, a0, a1, inv, cat, true, samples, A, lane, b, T.B, w);
  }
  float bv = -SM_INF;
  int bi = INT_MAX;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= A) continue;
    weights[(size_t)b * A + a] = w[j];
    const float v = inv[j] ? -SM_INF : w[j];
    if (beats(v, a, bv, bi)) {
      bv = v;
      bi = a;
    }
  }
  const int act = warp_argmax(bv, bi);
  if (lane == 0) action[b] = act;
}

// Tree.summary, tree.py:212-242
__global__ void summary_kernel(Tree T, float *visit, float2 *alpha, float2 *value_alpha, int8_t *q_out,
                               int32_t *q_dist, int8_t *v_out, int32_t *v_dist) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= T.B) return;
  const size_t ri = T.node(b, 0);
  const int player = T.to_play[ri];
  for (int a = lane; a < T.A; a += kWarp) {
    const size_t e = T.edge(b, 0, a), o = (size_t)b * T.A + a;
    const int8_t eo = T.edge_outcome[e];
    const int pay = T.edge_payload[e];
    const bool unresolved = eo == kNoOutcome;
    const int child = T.children[e];
    float2 al = T.edge_alpha[e];
    if (child != -1 && unresolved && pay <= 0 && T.ok(child)) {
      const size_t ci = T.node(b, child);
      al = align2(T.value_prior[ci], T.to_play[ci], player);
    }
    visit[o] = unresolved ? (float)pay : 0.0f;
    alpha[o] = al;
    q_out[o] = eo;
    q_dist[o] = unresolved ? -1 : pay;
  }
  if (lane == 0) {
    value_alpha[b] = T.value_alpha[ri];
    v_out[b] = T.node_outcome[ri];
    v_dist[b] = T.node_outcome[ri] == kNoOutcome ? -1 : T.node_payload[ri];
  }
}

template <int NS>
__global__ void __launch_bounds__(kThreads) prefix_cdf_kernel(const float2 *alpha, const uint8_t *invalid,
                                                              const int8_t *cat, int B, int A, PrefixParams P,
                                                              scacchi_prefix_out out) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  const PrefixScratch sc = prefix_scratch(2 * P.h + 1);
  if (b >= B) return;
  float a0[NS], a1[NS], policy[NS], raw[NS], dli[NS];
  bool inv[NS];
  int8_t oc[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const size_t i = (size_t)b * A + a;
    a0[j] = a1[j] = 1.0f;
    inv[j] = true;
    oc[j] = kNoOutcome;
    if (a >= A) continue;
    const float2 v = alpha[i];
    a0[j] = v.x;
    a1[j] = v.y;
    inv[j] = invalid[i] != 0;
    oc[j] = cat ? cat[i] : kNoOutcome;
  }
  PrefixLane L;
  warp_prefix_cdf<NS>(a0, a1, inv, oc, A, lane, P, sc, policy, raw, dli, L);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= A) continue;
    const size_t i = (size_t)b * A + a;
    out.policy[i] = policy[j];
    out.raw_policy[i] = raw[j];
    out.density_log_integral[i] = dli[j];
  }
  if (lane == 0) {
    out.raw_mass[b] = L.mass;
    out.normalization_error[b] = L.nerr;
    out.finite[b] = L.finite;
    out.grid_half_range[b] = L.hr;
    out.tail_range_clipped[b] = L.clipped;
    out.fallback_interval_count[b] = L.fic;
  }
}

template <int NS>
__global__ void __launch_bounds__(kThreads) mc_policy_kernel(const uint32_t *key, const float2 *alpha,
                                                             const uint8_t *invalid, const int8_t *cat, int B, int A,
                                                             int S, float *policy, int32_t *best_out) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= B) return;
  const sk_key k = {key[0], key[1]};
  float a0[NS], a1[NS], pol[NS];
  bool inv[NS];
  int8_t oc[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const size_t i = (size_t)b * A + a;
    a0[j] = a1[j] = 1.0f;
    inv[j] = true;
    oc[j] = kNoOutcome;
    if (a >= A) continue;
    const float2 v = alpha[i];
    a0[j] = v.x;
    a1[j] = v.y;
    inv[j] = invalid[i] != 0;
    oc[j] = cat ? cat[i] : kNoOutcome;
  }
  if (best_out) {
    const int best = warp_thompson<NS>(k, a0, a1, inv, oc, cat != nullptr, A, lane, (uint64_t)b * A * 2u,
                                       (uint64_t)B * A * 2u);
    if (lane == 0) best_out[b] = best;
    return;
  }
  warp_mc_policy<NS>(k, a0, a1, inv, oc, cat != nullptr, S, A, lane, b, B, pol);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a < A) policy[(size_t)b * A + a] = pol[j];
  }
}

template <int NS>
__global__ void __launch_bounds__(kThreads) update_context_kernel(const uint32_t *key, scacchi_context s, int B, int A,
                                                                  UpdateParams P, float2 *out_ea, int32_t *out_ep,
                                                                  float2 *out_va, uint8_t *out_unsafe) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  const PrefixScratch sc = prefix_scratch(2 * P.prefix.h + 1);
  if (b >= B) return;
  const sk_key k = {key[0], key[1]};
  NodeCtx<NS> c;
  c.active = s.active[b] != 0;
  c.leaf_active = s.leaf_active[b] != 0;
  c.leaf_action = s.leaf_action[b];
  c.leaf_value = reinterpret_cast<const float2 *>(s.leaf_value)[b];
  c.leaf_to_play = s.leaf_to_play[b];
  c.node_to_play = s.node_to_play[b];
  c.node_payload = s.node_payload[b];
  c.value_prior = reinterpret_cast<const float2 *>(s.value_prior)[b];
  c.value_alpha = reinterpret_cast<const float2 *>(s.value_alpha)[b];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const size_t i = (size_t)b * A + a;
    if (a >= A) {
      c.ea0[j] = c.ea1[j] = 1.0f;
      c.ep[j] = 0;
      c.eo[j] = kNoOutcome;
      c.inv[j] = true;
      c.cvis[j] = false;
      c.cprior[j] = c.cvalue[j] = make_float2(1.0f, 1.0f);
      c.cpay[j] = 0;
      c.cout[j] = kNoOutcome;
      c.ctp[j] = 0;
      continue;
    }
    const float2 ea = reinterpret_cast<const float2 *>(s.edge_alpha)[i];
    c.ea0[j] = ea.x;
    c.ea1[j] = ea.y;
    c.ep[j] = s.edge_payload[i];
    c.eo[j] = s.edge_outcome[i];
    c.inv[j] = s.invalid[i] != 0;
    c.cvis[j] = s.child_visited[i] != 0;
    c.cprior[j] = reinterpret_cast<const float2 *>(s.child_prior)[i];
    c.cvalue[j] = reinterpret_cast<const float2 *>(s.child_value)[i];
    c.cpay[j] = s.child_payload[i];
    c.cout[j] = s.child_outcome[i];
    c.ctp[j] = s.child_to_play[i];
  }
  NodeUpdate<NS> u;
  warp_posterior_update<NS>(k, c, A, lane, P, sc, b, B, u);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= A) continue;
    const size_t i = (size_t)b * A + a;
    out_ea[i] = make_float2(u.ea0[j], u.ea1[j]);
    out_ep[i] = u.ep[j];
  }
  if (lane == 0) {
    out_va[b] = u.value_alpha;
    out_unsafe[b] = u.unsafe;
  }
}

// _normalize_policy_on_support, play_search.py:263-295
template <int NS>
__device__ void warp_normalize_on_support(const float (&p)[NS], const bool (&support)[NS], int A, int lane,
                                          float temperature, float (&out)[NS]) {
  bool positive[NS];
  float masked[NS];
  int count = 0;
  bool anyp = false, mnan = false;
  float mx = -SM_INF;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const bool present = lane + kWarp * j < A;
    positive[j] = present && support[j] && p[j] > 0.0f;
    anyp |= positive[j];
    count += present && support[j];
    float c = p[j] > SM_TINY ? p[j] : SM_TINY;
    if (p[j] != p[j]) c = p[j];
    c = c < 1.0f ? c : 1.0f;
    masked[j] = positive[j] ? sm_logf(c) : SM_FMIN;
    if (present) {
      mnan |= masked[j] != masked[j];
      if (masked[j] > mx) mx = masked[j];
    }
  }
  mx = warp_max_float(mx);
  if (__any_sync(kFull, mnan)) mx = SM_NAN;
  const bool has_positive = __any_sync(kFull, anyp);
  count = __reduce_add_sync(kFull, count);
  float scaled[NS];
  float smax = -SM_INF;
  bool snan = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    scaled[j] = positive[j] ? (masked[j] - mx) / temperature : SM_FMIN;
    if (lane + kWarp * j < A) {
      snan |= scaled[j] != scaled[j];
      if (scaled[j] > smax) smax = scaled[j];
    }
  }
  smax = warp_max_float(smax);
  if (__any_sync(kFull, snan)) smax = SM_NAN;
  float e[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) e[j] = sm_expf(scaled[j] - smax);
  const float total = warp_sum<NS>(e, A, lane);
  const float den = (float)(count > 1 ? count : 1);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const float nrm = positive[j] ? e[j] / total : 0.0f;
    out[j] = has_positive ? nrm : (support[j] ? 1.0f : 0.0f) / den;
  }
}

// _dirichlet_root_policy_readout, play_search.py:298-364
template <int NS>
__global__ void __launch_bounds__(kThreads) root_readout_kernel(int B, int A, const float *native, const float *visit,
                                                                const float2 *alpha, const int8_t *q_out,
                                                                const int32_t *q_dist, const int8_t *v_out,
                                                                const uint8_t *legal, int search_evidence,
                                                                float temperature, PrefixParams P, float *target,
                                                                uint8_t *accepted_out) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  const PrefixScratch sc = prefix_scratch(2 * P.h + 1);
  if (b >= B) return;
  bool lg[NS], support[NS], inv[NS];
  float nat[NS], a0[NS], a1[NS];
  int8_t qo[NS];
  bool any_cand = false, any_legal = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const size_t i = (size_t)b * A + a;
    lg[j] = false;
    nat[j] = 0.0f;
    a0[j] = a1[j] = 1.0f;
    qo[j] = kNoOutcome;
    support[j] = false;
    if (a >= A) continue;
    lg[j] = legal[i] != 0;
    nat[j] = native[i];
    const float2 v = alpha[i];
    a0[j] = v.x;
    a1[j] = v.y;
    qo[j] = q_out[i];
    support[j] = lg[j] && (visit[i] > 0.0f || qo[j] != kNoOutcome);
    any_cand |= support[j];
    any_legal |= lg[j];
  }
  const bool has_candidate = __any_sync(kFull, any_cand);
  const bool has_legal = __any_sync(kFull, any_legal);
  bool any_support = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    if (!search_evidence || !has_candidate) support[j] = lg[j];
    inv[j] = !support[j];
    any_support |= support[j] && lane + kWarp * j < A;
  }
  const bool has_support = __any_sync(kFull, any_support);
  float pol[NS];
  warp_normalize_on_support<NS>(nat, support, A, lane, 1.0f, pol);
  float est[NS], raw[NS], dli[NS];
  PrefixLane L;
  warp_prefix_cdf<NS>(a0, a1, inv, qo, A, lane, P, sc, est, raw, dli, L);
  float derr = 0.0f;
  bool dnan = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    if (lane + kWarp * j >= A) continue;
    const float v = fabsf(dli[j]);
    dnan |= v != v;
    if (v > derr) derr = v;
  }
  derr = warp_max_float(derr);
  dnan = __any_sync(kFull, dnan);
  const bool unsafe = L.clipped || !L.finite || (!dnan && derr > 0.01f);
  const int8_t vo = v_out[b];
  const bool root_cat = vo != kNoOutcome;
  const bool accepted = has_support && !root_cat && !unsafe;
  float tgt[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) tgt[j] = accepted ? est[j] : pol[j];
  // categorical_action_population, action_selection.py:62-75
  float score[NS];
  float best = -SM_INF;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    score[j] = -SM_INF;
    if (a >= A) continue;
    const bool legal_s = !inv[j];
    const float dist = (float)q_dist[(size_t)b * A + a];
    if (vo == 1) score[j] = (legal_s && qo[j] == 1) ? -dist : -SM_INF;
    else if (vo == 0) score[j] = (legal_s && qo[j] == 0) ? dist : -SM_INF;
    else score[j] = (legal_s && qo[j] == 1) ? 0.0f : -SM_INF;
    if (score[j] > best) best = score[j];
  }
  best = warp_max_float(best);
  int count = 0;
  bool tied[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    tied[j] = lane + kWarp * j < A && sm_isfinite(score[j]) && score[j] == best;
    count += tied[j];
  }
  count = __reduce_add_sync(kFull, count);
  const float cden = (float)(count > 1 ? count : 1);
  float cat[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) cat[j] = (tied[j] ? 1.0f : 0.0f) / cden;
  const float cat_sum = warp_sum<NS>(cat, A, lane);
  if (root_cat && has_legal && cat_sum > 0.0f) {
#pragma unroll
    for (int j = 0; j < NS; ++j) tgt[j] = cat[j];
  }
  float fin[NS];
  warp_normalize_on_support<NS>(tgt, support, A, lane, temperature, fin);
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a < A) target[(size_t)b * A + a] = fin[j];
  }
  if (lane == 0 && accepted_out) accepted_out[b] = accepted;
}

// _dirichlet_commitment_policy (play_search.py:627-705): the root policy an
// action is committed from.  `sampled` is posterior_best_policy over the
// commitment support (computed by the caller with the commitment key);
// a categorical root takes the one-hot of the search action instead.  The
// native policy is normalised on the support; with the numerical update
// the Q21 estimate replaces it where it is safe (_numerical_policy_readout,
// play_search.py:161-229).
template <int NS>
__global__ void __launch_bounds__(kThreads) commitment_kernel(int B, int A, const float *sampled,
                                                              const int32_t *search_action, const float2 *alpha,
                                                              const int8_t *q_out, const int8_t *v_out,
                                                              const uint8_t *legal, const uint8_t *evidence,
                                                              int search_evidence, int numerical, PrefixParams P,
                                                              float *policy) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  const PrefixScratch sc = prefix_scratch(2 * P.h + 1);
  if (b >= B) return;
  const bool root_cat = v_out[b] != kNoOutcome;
  const int solved = search_action[b];
  bool lg[NS], support[NS], inv[NS];
  float nat[NS], a0[NS], a1[NS];
  int8_t qo[NS];
  bool any_cand = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const size_t i = (size_t)b * A + a;
    lg[j] = support[j] = false;
    nat[j] = 0.0f;
    a0[j] = a1[j] = 1.0f;
    qo[j] = kNoOutcome;
    if (a >= A) continue;
    lg[j] = legal[i] != 0;
    qo[j] = q_out[i];
    const float2 v = alpha[i];
    a0[j] = v.x;
    a1[j] = v.y;
    nat[j] = root_cat ? (a == solved ? 1.0f : 0.0f) : sampled[i];
    // _root_policy_support, play_search.py:232-252
    support[j] = lg[j] && (evidence[i] != 0 || qo[j] != kNoOutcome);
    any_cand |= support[j];
  }
  const bool has_candidate = __any_sync(kFull, any_cand);
  bool any_support = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    if (!search_evidence || !has_candidate) support[j] = lg[j];
    inv[j] = !support[j];
    any_support |= support[j] && lane + kWarp * j < A;
  }
  const bool has_support = __any_sync(kFull, any_support);
  float out[NS];
  warp_normalize_on_support<NS>(nat, support, A, lane, 1.0f, out);
  if (numerical) {
    float est[NS], raw[NS], dli[NS];
    PrefixLane L;
    warp_prefix_cdf<NS>(a0, a1, inv, qo, A, lane, P, sc, est, raw, dli, L);
    float derr = 0.0f;
    bool dnan = false;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      if (lane + kWarp * j >= A) continue;
      const float v = fabsf(dli[j]);
      dnan |= v != v;
      if (v > derr) derr = v;
    }
    derr = warp_max_float(derr);
    dnan = __any_sync(kFull, dnan);
    const bool unsafe = L.clipped || !L.finite || (!dnan && derr > 0.01f);
    if (has_support && !root_cat && !unsafe) {
#pragma unroll
      for (int j = 0; j < NS; ++j) out[j] = est[j];
    }
  }
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a < A) policy[(size_t)b * A + a] = out[j];
  }
}

// posterior_best_action / posterior_sample_action
// (dirichlet_q_search.py:79-116): kind 0 takes the masked argmax, kind 1
// samples jax.random.categorical(key, logits) = argmax(logits + Gumbel
// noise) of the power-temperature logits log(clip(p, 1e-8, 1)) / T over the
// legal actions with positive policy (all legal actions if none has).
template <int NS>
__global__ void __launch_bounds__(kThreads) commit_action_kernel(int kind, const uint32_t *key_words,
                                                                 const float *policy, const uint8_t *legal, int B,
                                                                 int A, float temperature, int32_t *action) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= B) return;
  const sk_key key = kind == 1 ? sk_key{key_words[0], key_words[1]} : sk_key{0u, 0u};
  float p[NS];
  bool lg[NS], pos[NS];
  bool any_pos = false;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    const size_t i = (size_t)b * A + a;
    p[j] = a < A ? policy[i] : 0.0f;
    lg[j] = a < A && legal[i] != 0;
    pos[j] = lg[j] && p[j] > 0.0f;
    any_pos |= pos[j];
  }
  any_pos = __any_sync(kFull, any_pos);
  float bv = -SM_INF;
  int bi = INT_MAX;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= A) continue;
    float score;
    if (kind == 0) {
      score = lg[j] ? p[j] : -SM_INF;
    } else {
      const bool eligible = any_pos ? pos[j] : lg[j];
      float c = p[j] > 1e-8f ? p[j] : 1e-8f;
      if (p[j] != p[j]) c = p[j];
      c = c < 1.0f ? c : 1.0f;
      const float logit = eligible ? sm_logf(c) / temperature : SM_FMIN;
      // jax.random.gumbel: -log(-log(uniform(key, [B, A], tiny, 1)))
      const float u = sk_uniform(key, (uint64_t)b * A + a, SM_TINY, 1.0f);
      score = logit + (-sm_logf(-sm_logf(u)));
    }
    if (beats(score, a, bv, bi)) {
      bv = score;
      bi = a;
    }
  }
  const int best = warp_argmax(bv, bi);
  if (lane == 0) action[b] = best;
}

// ------------------------------------------------------------------------
// synthetic game
// ------------------------------------------------------------------------

template <int NS>
__device__ void synthetic_eval(const se_params &p, se_state s, int b, int lane, float2 *value, float2 *av,
                               uint8_t *inv, float *logits) {
  const int A = p.num_actions;
  const int deg = se_degenerate_lane(&p, b);
  bool invalid[NS];
  bool any_legal = false;
  float uv = SM_INF;
  int ui = INT_MAX;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    invalid[j] = true;
    if (a >= A) continue;
    const float u = se_legal_u(s, a);
    invalid[j] = !(u < p.legal_prob);
    any_legal |= !invalid[j];
    if (u < uv || (u == uv && a < ui)) {
      uv = u;
      ui = a;
    }
  }
  if (!__any_sync(kFull, any_legal)) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ou = __shfl_xor_sync(kFull, uv, off);
      const int oi = __shfl_xor_sync(kFull, ui, off);
      if (ou < uv || (ou == uv && oi < ui)) {
        uv = ou;
        ui = oi;
      }
    }
#pragma unroll
    for (int j = 0; j < NS; ++j)
      if (lane + kWarp * j == ui) invalid[j] = false;
  }
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int a = lane + kWarp * j;
    if (a >= A) continue;
    const size_t i = (size_t)b * A + a;
    inv[i] = invalid[j];
    av[i] = make_float2(se_q_alpha(&p, s, a, 0, deg), se_q_alpha(&p, s, a, 1, deg));
    if (logits) logits[i] = se_logit(s, a);
  }
  if (lane == 0) value[b] = make_float2(se_value_alpha(&p, s, 0, deg), se_value_alpha(&p, s, 1, deg));
}

template <int NS>
__global__ void __launch_bounds__(kThreads) synthetic_root_kernel(se_params p, int B, float *logits, float2 *value,
                                                                  float2 *av, uint8_t *inv, int8_t *term,
                                                                  int32_t *tp, se_state *emb) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= B) return;
  const se_state s = se_root_state(&p, b);
  synthetic_eval<NS>(p, s, b, lane, value, av, inv, logits);
  if (lane == 0) {
    term[b] = (int8_t)se_terminal(&p, s);
    tp[b] = s.to_play;
    emb[b] = s;
  }
}

template <int NS>
__global__ void __launch_bounds__(kThreads) synthetic_evaluate_kernel(se_params p, int B, const se_state *states,
                                                                      float *logits, float2 *value, float2 *av,
                                                                      uint8_t *inv, int8_t *term, int32_t *tp) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= B) return;
  const se_state s = states[b];
  synthetic_eval<NS>(p, s, b, lane, value, av, inv, logits);
  if (lane == 0) {
    term[b] = (int8_t)se_terminal(&p, s);
    tp[b] = s.to_play;
  }
}

template <int NS>
__global__ void __launch_bounds__(kThreads) synthetic_recurrent_kernel(se_params p, int B, const int32_t *action,
                                                                       const se_state *parent, float2 *value,
                                                                       float2 *av, uint8_t *inv, int8_t *term,
                                                                       int32_t *tp, se_state *child) {
  const int b = warp_lane_index(), lane = threadIdx.x % kWarp;
  if (b >= B) return;
  const se_state s = se_child_state(parent[b], action[b]);
  synthetic_eval<NS>(p, s, b, lane, value, av, inv, nullptr);
  if (lane == 0) {
    term[b] = (int8_t)se_terminal(&p, s);
    tp[b] = s.to_play;
    child[b] = s;
  }
}

// ------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }
inline int blocks_for(int lanes) { return (lanes + kWarpsPerBlock - 1) / kWarpsPerBlock; }
inline int slots_for(int A) { return (A + kWarp - 1) / kWarp; }

inline int launched() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaPeekAtLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

bool tree_ok(const scacchi_tree *t) {
  if (!t || t->batch < 0 || t->num_nodes < 1 || t->num_actions < 1 || t->num_actions > 128) return false;
  if (t->action_stride < t->num_actions || t->emb_bytes < 0) return false;
  if (t->batch > 0 && (!t->parents || !t->children_index || !t->node_to_play || !t->node_outcome ||
                       !t->node_payload || !t->edge_outcome || !t->edge_payload || !t->node_value_prior ||
                       !t->node_value_alpha || !t->edge_alpha || !t->invalid))
    return false;
  if (t->emb_bytes > 0 && !t->embedding) return false;
  return true;
}

bool params_ok(const scacchi_update_params *p) {
  if (!p || (p->rule != 0 && p->rule != 1) || p->samples < 1) return false;
  if (p->rule == 1 && (p->half_width < 1 || p->half_width > kMaxHalfWidth)) return false;
  return true;
}

constexpr size_t kCtaSmemLimit = 160 * 1024;

size_t prefix_smem(int half_width) { return (size_t)kWarpsPerBlock * 6 * (2 * half_width + 1) * sizeof(float); }

// Dynamic shared memory above 48 KB needs an opt-in; the CTA-per-lane
// kernels also ask for the largest shared-memory carveout, so their
// residency is set by registers and shared memory, not by the L1 split.
template <typename K>
void allow_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}

#define SCACCHI_DISPATCH(A, ...)                          \
  switch (slots_for(A)) {                                 \
    case 1: { constexpr int NS = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int NS = 2; __VA_ARGS__; } break; \
    case 3: { constexpr int NS = 3; __VA_ARGS__; } break; \
    default: { constexpr int NS = 4; __VA_ARGS__; } break; \
  }

se_params make_se(const scacchi_synthetic_params *p) {
  se_params s;
  s.seed_k0 = p->seed_k0;
  s.seed_k1 = p->seed_k1;
  s.num_actions = p->num_actions;
  s.legal_prob = p->legal_prob;
  s.terminal_prob = p->terminal_prob;
  s.degenerate_lane_prob = p->degenerate_lane_prob;
  s.degenerate_alpha = p->degenerate_alpha;
  s.logc_mean = p->logc_mean;
  s.logc_std = p->logc_std;
  s.logc_min = p->logc_min;
  s.logc_max = p->logc_max;
  return s;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

// ==========================================================================
// C ABI
// ==========================================================================

extern "C" {

int scacchi_tree_init(const scacchi_tree *tree, const float *root_value, const float *root_action_values,
                      const uint8_t *root_invalid, const int8_t *root_terminal, const int32_t *root_to_play,
                      const uint8_t *root_embedding, int32_t full_init, void *stream) {
  if (!tree_ok(tree) || !root_value || !root_action_values || !root_invalid || !root_terminal || !root_to_play)
    return SCACCHI_EINVAL;
  if (tree->batch == 0) return SCACCHI_OK;
  Tree T = make_tree(tree);
  tree_init_kernel<<<blocks_for(T.B), kThreads, 0, as_stream(stream)>>>(
      T, reinterpret_cast<const float2 *>(root_value), reinterpret_cast<const float2 *>(root_action_values),
      root_invalid, root_terminal, root_to_play, root_embedding, full_init);
  return launched();
}

int scacchi_simulate(const scacchi_tree *tree, const uint32_t *simulate_key, int32_t max_depth, int32_t *parent,
                     int32_t *action, uint8_t *active, uint8_t *parent_embedding, uint64_t *stats, void *stream) {
  if (!tree_ok(tree) || !simulate_key || !parent || !action || !active || max_depth < 1) return SCACCHI_EINVAL;
  if (tree->batch == 0) return SCACCHI_OK;
  Tree T = make_tree(tree);
  uint8_t *pe = T.E > 0 ? parent_embedding : nullptr;
  SCACCHI_DISPATCH(T.A, {
    const size_t smem = cta_smem_floats<NS>(1) * sizeof(float);
    allow_smem(simulate_cta_kernel<NS>, smem);
    simulate_cta_kernel<NS><<<T.B, 32 * NS, smem, as_stream(stream)>>>(
        T, simulate_key, max_depth, parent, action, active, pe, reinterpret_cast<unsigned long long *>(stats));
  });
  return launched();
}

int scacchi_expand(const scacchi_tree *tree, int32_t new_node, const int32_t *parent, const int32_t *action,
                   const uint8_t *active, const float *step_value, const float *step_action_values,
                   const uint8_t *step_invalid, const int8_t *step_terminal, const int32_t *step_to_play,
                   const uint8_t *child_embedding, int32_t lazy_init, void *stream) {
  if (!tree_ok(tree) || !parent || !action || !active || !step_value || !step_action_values || !step_invalid ||
      !step_terminal || !step_to_play)
    return SCACCHI_EINVAL;
  if (tree->batch == 0) return SCACCHI_OK;
  Tree T = make_tree(tree);
  expand_kernel<<<blocks_for(T.B), kThreads, 0, as_stream(stream)>>>(
      T, new_node, parent, action, active, reinterpret_cast<const float2 *>(step_value),
      reinterpret_cast<const float2 *>(step_action_values), step_invalid, step_terminal, step_to_play,
      T.E > 0 ? child_embedding : nullptr, lazy_init);
  return launched();
}

int scacchi_backward(const scacchi_tree *tree, const uint32_t *backward_key, const int32_t *parent,
                     const int32_t *action, const uint8_t *active, const float *step_value,
                     const int32_t *step_to_play, const scacchi_update_params *params, uint64_t *stats,
                     void *stream) {
  if (!tree_ok(tree) || !backward_key || !parent || !action || !active || !step_value || !step_to_play ||
      !params_ok(params))
    return SCACCHI_EINVAL;
  if (tree->batch == 0) return SCACCHI_OK;
  Tree T = make_tree(tree);
  const UpdateParams P = make_params(params);
  const int Q = P.rule == 1 ? 2 * P.prefix.h + 1 : 1;
  SCACCHI_DISPATCH(T.A, {
    const size_t smem = cta_smem_floats<NS>(Q) * sizeof(float);
    if (smem <= kCtaSmemLimit) {
      auto launch = [&](auto kernel) {
        allow_smem(kernel, smem);
        kernel<<<T.B, 32 * NS, smem, as_stream(stream)>>>(T, backward_key, parent, action, active,
                                                           reinterpret_cast<const float2 *>(step_value),
                                                           step_to_play, P,
                                                           reinterpret_cast<unsigned long long *>(stats));
      };
      if (P.rule == 1) launch(backward_cta_kernel<NS, 1>);
      else launch(backward_cta_kernel<NS, 0>);
    } else {
      // very fine grids: the warp-per-lane kernel recomputes instead of
      // holding [Q][A] matrices in shared memory
      const size_t wsmem = prefix_smem(P.rule == 1 ? P.prefix.h : 1);
      allow_smem(backward_kernel<NS>, wsmem);
      backward_kernel<NS><<<blocks_for(T.B), kThreads, wsmem, as_stream(stream)>>>(
          T, backward_key, parent, action, active, reinterpret_cast<const float2 *>(step_value), step_to_play, P,
          reinterpret_cast<unsigned long long *>(stats));
    }
  });
  return launched();
}

int scacchi_root_policy(const scacchi_tree *tree, const uint32_t *policy_key, const uint8_t *invalid,
                        int32_t policy_samples, float *action_weights, int32_t *action, void *stream) {
  if (!tree_ok(tree) || !policy_key || !invalid || !action_weights || !action) return SCACCHI_EINVAL;
  if (tree->batch == 0) return SCACCHI_OK;
  Tree T = make_tree(tree);
  const int S = policy_samples > 1 ? policy_samples : 1;
  SCACCHI_DISPATCH(T.A, (root_policy_kernel<NS><<<blocks_for(T.B), kThreads, 0, as_stream(stream)>>>(
                               T, policy_key, invalid, S, action_weights, action)));
  return launched();
}

int scacchi_summary(const scacchi_tree *tree, float *visit_counts, float *alpha, float *value_alpha,
                    int8_t *q_outcome, int32_t *q_distance, int8_t *v_outcome, int32_t *v_distance,
                    void *stream) {
  if (!tree_ok(tree) || !visit_counts || !alpha || !value_alpha || !q_outcome || !q_distance || !v_outcome ||
      !v_distance)
    return SCACCHI_EINVAL;
  if (tree->batch == 0) return SCACCHI_OK;
  Tree T = make_tree(tree);
  summary_kernel<<<blocks_for(T.B), kThreads, 0, as_stream(stream)>>>(
      T, visit_counts, reinterpret_cast<float2 *>(alpha), reinterpret_cast<float2 *>(value_alpha), q_outcome,
      q_distance, v_outcome, v_distance);
  return launched();
}

int scacchi_prefix_cdf(const float *alpha, const uint8_t *invalid, const int8_t *categorical_outcome, int32_t batch,
                       int32_t num_actions, int32_t half_width, float tail_scale, float min_half_range,
                       float max_half_range, const scacchi_prefix_out *out, void *stream) {
  if (!alpha || !invalid || !out || batch < 0 || num_actions < 1 || num_actions > 128 || half_width < 1 ||
      half_width > kMaxHalfWidth || !out->policy || !out->raw_policy || !out->raw_mass ||
      !out->normalization_error || !out->finite || !out->grid_half_range || !out->tail_range_clipped ||
      !out->density_log_integral || !out->fallback_interval_count)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  PrefixParams P{half_width, tail_scale, min_half_range, max_half_range};
  const size_t smem = prefix_smem(half_width);
  SCACCHI_DISPATCH(num_actions, {
    allow_smem(prefix_cdf_kernel<NS>, smem);
    prefix_cdf_kernel<NS><<<blocks_for(batch), kThreads, smem, as_stream(stream)>>>(
        reinterpret_cast<const float2 *>(alpha), invalid, categorical_outcome, batch, num_actions, P, *out);
  });
  return launched();
}

int scacchi_posterior_best_policy(const uint32_t *key, const float *alpha, const uint8_t *invalid,
                                  const int8_t *categorical_outcome, int32_t batch, int32_t num_actions,
                                  int32_t num_samples, float *policy, void *stream) {
  if (!key || !alpha || !invalid || !policy || batch < 0 || num_actions < 1 || num_actions > 128 || num_samples < 1)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  SCACCHI_DISPATCH(num_actions, (mc_policy_kernel<NS><<<blocks_for(batch), kThreads, 0, as_stream(stream)>>>(
                                    key, reinterpret_cast<const float2 *>(alpha), invalid, categorical_outcome, batch,
                                    num_actions, num_samples, policy, nullptr)));
  return launched();
}

int scacchi_thompson_sample(const uint32_t *key, const float *alpha, const uint8_t *invalid,
                            const int8_t *categorical_outcome, int32_t batch, int32_t num_actions, int32_t *action,
                            void *stream) {
  if (!key || !alpha || !invalid || !action || batch < 0 || num_actions < 1 || num_actions > 128)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  SCACCHI_DISPATCH(num_actions, (mc_policy_kernel<NS><<<blocks_for(batch), kThreads, 0, as_stream(stream)>>>(
                                    key, reinterpret_cast<const float2 *>(alpha), invalid, categorical_outcome, batch,
                                    num_actions, 1, nullptr, action)));
  return launched();
}

int scacchi_update_posterior(const uint32_t *key, const scacchi_context *context, int32_t batch, int32_t num_actions,
                             const scacchi_update_params *params, float *edge_alpha, int32_t *edge_payload,
                             float *value_alpha, uint8_t *unsafe, void *stream) {
  if (!key || !context || !params_ok(params) || !edge_alpha || !edge_payload || !value_alpha || !unsafe ||
      batch < 0 || num_actions < 1 || num_actions > 128)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  const UpdateParams P = make_params(params);
  const size_t smem = prefix_smem(P.rule == 1 ? P.prefix.h : 1);
  SCACCHI_DISPATCH(num_actions, {
    allow_smem(update_context_kernel<NS>, smem);
    update_context_kernel<NS><<<blocks_for(batch), kThreads, smem, as_stream(stream)>>>(
        key, *context, batch, num_actions, P, reinterpret_cast<float2 *>(edge_alpha), edge_payload,
        reinterpret_cast<float2 *>(value_alpha), unsafe);
  });
  return launched();
}

int scacchi_root_readout(int32_t batch, int32_t num_actions, const float *native_policy, const float *visit_counts,
                         const float *alpha, const int8_t *q_outcome, const int32_t *q_distance,
                         const int8_t *v_outcome, const uint8_t *legal, int32_t search_evidence_support,
                         float temperature, int32_t half_width, float tail_scale, float min_half_range,
                         float max_half_range, float *policy_target, uint8_t *accepted, void *stream) {
  if (!native_policy || !visit_counts || !alpha || !q_outcome || !q_distance || !v_outcome || !legal ||
      !policy_target || batch < 0 || num_actions < 1 || num_actions > 128 || half_width < 1 ||
      half_width > kMaxHalfWidth)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  PrefixParams P{half_width, tail_scale, min_half_range, max_half_range};
  const size_t smem = prefix_smem(half_width);
  SCACCHI_DISPATCH(num_actions, {
    allow_smem(root_readout_kernel<NS>, smem);
    root_readout_kernel<NS><<<blocks_for(batch), kThreads, smem, as_stream(stream)>>>(
        batch, num_actions, native_policy, visit_counts, reinterpret_cast<const float2 *>(alpha), q_outcome,
        q_distance, v_outcome, legal, search_evidence_support, temperature, P, policy_target, accepted);
  });
  return launched();
}

int scacchi_commitment_policy(int32_t batch, int32_t num_actions, const float *sampled_policy,
                              const int32_t *search_action, const float *alpha, const int8_t *q_outcome,
                              const int8_t *v_outcome, const uint8_t *legal, const uint8_t *positive_evidence,
                              int32_t search_evidence_support, int32_t numerical, int32_t half_width,
                              float tail_scale, float min_half_range, float max_half_range, float *policy,
                              void *stream) {
  if (!sampled_policy || !search_action || !alpha || !q_outcome || !v_outcome || !legal || !positive_evidence ||
      !policy || batch < 0 || num_actions < 1 || num_actions > 128 || half_width < 1 || half_width > kMaxHalfWidth)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  PrefixParams P{half_width, tail_scale, min_half_range, max_half_range};
  const size_t smem = prefix_smem(half_width);
  SCACCHI_DISPATCH(num_actions, {
    allow_smem(commitment_kernel<NS>, smem);
    commitment_kernel<NS><<<blocks_for(batch), kThreads, smem, as_stream(stream)>>>(
        batch, num_actions, sampled_policy, search_action, reinterpret_cast<const float2 *>(alpha), q_outcome,
        v_outcome, legal, positive_evidence, search_evidence_support, numerical, P, policy);
  });
  return launched();
}

int scacchi_commit_action(int32_t kind, const uint32_t *key, const float *policy, const uint8_t *legal,
                          int32_t batch, int32_t num_actions, float temperature, int32_t *action, void *stream) {
  if ((kind != 0 && kind != 1) || !policy || !legal || !action || batch < 0 || num_actions < 1 ||
      num_actions > 128 || (kind == 1 && (!key || !(temperature > 0.0f) || !sm_isfinite(temperature))))
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  SCACCHI_DISPATCH(num_actions, (commit_action_kernel<NS><<<blocks_for(batch), kThreads, 0, as_stream(stream)>>>(
                                    kind, key, policy, legal, batch, num_actions, temperature, action)));
  return launched();
}

int scacchi_synthetic_root(const scacchi_synthetic_params *params, int32_t batch, float *prior_logits, float *value,
                           float *action_values, uint8_t *invalid, int8_t *terminal, int32_t *to_play,
                           uint8_t *embedding, void *stream) {
  if (!params || params->num_actions < 1 || params->num_actions > 128 || batch < 0 || !prior_logits || !value ||
      !action_values || !invalid || !terminal || !to_play || !embedding)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  const se_params p = make_se(params);
  SCACCHI_DISPATCH(p.num_actions, (synthetic_root_kernel<NS><<<blocks_for(batch), kThreads, 0, as_stream(stream)>>>(
                                       p, batch, prior_logits, reinterpret_cast<float2 *>(value),
                                       reinterpret_cast<float2 *>(action_values), invalid, terminal, to_play,
                                       reinterpret_cast<se_state *>(embedding))));
  return launched();
}

int scacchi_synthetic_evaluate(const scacchi_synthetic_params *params, int32_t batch, const uint8_t *states,
                               float *prior_logits, float *value, float *action_values, uint8_t *invalid,
                               int8_t *terminal, int32_t *to_play, void *stream) {
  if (!params || params->num_actions < 1 || params->num_actions > 128 || batch < 0 || !states || !prior_logits ||
      !value || !action_values || !invalid || !terminal || !to_play)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  const se_params p = make_se(params);
  SCACCHI_DISPATCH(p.num_actions,
                   (synthetic_evaluate_kernel<NS><<<blocks_for(batch), kThreads, 0, as_stream(stream)>>>(
                       p, batch, reinterpret_cast<const se_state *>(states), prior_logits,
                       reinterpret_cast<float2 *>(value), reinterpret_cast<float2 *>(action_values), invalid,
                       terminal, to_play)));
  return launched();
}

int scacchi_synthetic_recurrent(const scacchi_synthetic_params *params, int32_t batch, const int32_t *action,
                                const uint8_t *parent_embedding, float *value, float *action_values, uint8_t *invalid,
                                int8_t *terminal, int32_t *to_play, uint8_t *child_embedding, void *stream) {
  if (!params || params->num_actions < 1 || params->num_actions > 128 || batch < 0 || !action || !parent_embedding ||
      !value || !action_values || !invalid || !terminal || !to_play || !child_embedding)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  const se_params p = make_se(params);
  SCACCHI_DISPATCH(p.num_actions,
                   (synthetic_recurrent_kernel<NS><<<blocks_for(batch), kThreads, 0, as_stream(stream)>>>(
                       p, batch, action, reinterpret_cast<const se_state *>(parent_embedding),
                       reinterpret_cast<float2 *>(value), reinterpret_cast<float2 *>(action_values), invalid,
                       terminal, to_play, reinterpret_cast<se_state *>(child_embedding))));
  return launched();
}

size_t scacchi_search_workspace_bytes(int32_t batch, int32_t num_actions, int32_t emb_bytes) {
  const size_t B = batch > 0 ? (size_t)batch : 0, A = num_actions > 0 ? (size_t)num_actions : 0;
  const size_t E = emb_bytes > 0 ? (size_t)emb_bytes : 0;
  return align256(B * 4) * 2 + align256(B) + align256(B * E) * 2 + align256(B * 8) + align256(B * A * 8) +
         align256(B * A) + align256(B) + align256(B * 4);
}

int scacchi_search_synthetic(const scacchi_tree *tree, const scacchi_synthetic_params *env, const uint32_t *keys,
                             int32_t num_simulations, int32_t max_depth, const scacchi_update_params *params,
                             void *workspace, uint64_t *stats, void *stream) {
  if (!tree_ok(tree) || !env || !keys || num_simulations < 0 || max_depth < 1 || !params_ok(params) ||
      !workspace || env->num_actions != tree->num_actions || tree->emb_bytes != (int32_t)sizeof(se_state) ||
      num_simulations + 1 > tree->num_nodes)
    return SCACCHI_EINVAL;
  const int B = tree->batch, A = tree->num_actions, E = tree->emb_bytes;
  if (B == 0) return SCACCHI_OK;
  uint8_t *w = static_cast<uint8_t *>(workspace);
  auto take = [&w](size_t bytes) {
    uint8_t *p = w;
    w += align256(bytes);
    return p;
  };
  int32_t *parent = reinterpret_cast<int32_t *>(take((size_t)B * 4));
  int32_t *action = reinterpret_cast<int32_t *>(take((size_t)B * 4));
  uint8_t *active = take(B);
  uint8_t *pemb = take((size_t)B * E);
  uint8_t *cemb = take((size_t)B * E);
  float *value = reinterpret_cast<float *>(take((size_t)B * 8));
  float *av = reinterpret_cast<float *>(take((size_t)B * A * 8));
  uint8_t *inv = take((size_t)B * A);
  int8_t *term = reinterpret_cast<int8_t *>(take(B));
  int32_t *tp = reinterpret_cast<int32_t *>(take((size_t)B * 4));
  for (int i = 0; i < num_simulations; ++i) {
    const uint32_t *k = keys + (size_t)i * 8;
    int rc = scacchi_simulate(tree, k + 2, max_depth, parent, action, active, pemb, stats ? stats + 4 : nullptr,
                              stream);
    if (rc) return rc;
    rc = scacchi_synthetic_recurrent(env, B, action, pemb, value, av, inv, term, tp, cemb, stream);
    if (rc) return rc;
    rc = scacchi_expand(tree, i + 1, parent, action, active, value, av, inv, term, tp, cemb, 1, stream);
    if (rc) return rc;
    rc = scacchi_backward(tree, k + 6, parent, action, active, value, tp, params, stats, stream);
    if (rc) return rc;
  }
  return SCACCHI_OK;
}

int scacchi_device_error(uint32_t *flags) {
  if (!flags) return SCACCHI_EINVAL;
  uint32_t v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_error_flags, sizeof(v)) != cudaSuccess) return SCACCHI_ECUDA;
  if (cudaMemcpyToSymbol(g_error_flags, &zero, sizeof(zero)) != cudaSuccess) return SCACCHI_ECUDA;
  *flags = v;
  return SCACCHI_OK;
}

uint64_t scacchi_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

}  // extern "C"

// ==========================================================================
// host-side key schedule (no device work)
// ==========================================================================

extern "C" {

/* search.py:207-209: key_{i+1}, simulate, expand, backward = split(key_i, 4)
 * for i < num_simulations, starting from key_0 = search key.  out is
 * uint32[num_simulations, 4, 2]. */
int scacchi_key_schedule(uint32_t k0, uint32_t k1, int32_t num_simulations, uint32_t *out) {
  if (num_simulations < 0 || (!out && num_simulations > 0)) return SCACCHI_EINVAL;
  sk_key key = {k0, k1};
  for (int i = 0; i < num_simulations; ++i) {
    for (int j = 0; j < 4; ++j) {
      const sk_key s = sk_split(key, (uint64_t)j);
      out[(size_t)i * 8 + 2 * j] = s.k0;
      out[(size_t)i * 8 + 2 * j + 1] = s.k1;
    }
    key = sk_split(key, 0);
  }
  return SCACCHI_OK;
}

/* jax.random.split(key, n) -> uint32[n, 2] and fold_in(key, d) on the host. */
int scacchi_split_host(uint32_t k0, uint32_t k1, int32_t n, uint32_t *out) {
  if (n < 0 || (!out && n > 0)) return SCACCHI_EINVAL;
  const sk_key key = {k0, k1};
  for (int i = 0; i < n; ++i) {
    const sk_key s = sk_split(key, (uint64_t)i);
    out[2 * i] = s.k0;
    out[2 * i + 1] = s.k1;
  }
  return SCACCHI_OK;
}

int scacchi_fold_in_host(uint32_t k0, uint32_t k1, uint32_t data, uint32_t *out) {
  if (!out) return SCACCHI_EINVAL;
  const sk_key s = sk_fold_in(sk_key{k0, k1}, data);
  out[0] = s.k0;
  out[1] = s.k1;
  return SCACCHI_OK;
}

}  // extern "C"

// ==========================================================================
// Synthetic-game search with library-owned scratch (no allocation per call)
// ==========================================================================
//
// Some callers cannot allocate device memory at call time.  The main one is
// an XLA FFI handler: it runs inside XLA, whose allocator has usually
// reserved most of the device's memory up front and hands out scratch only
// as buffers declared in the call's signature, so a cudaMalloc there can
// fail, or synchronise the device in the middle of XLA's stream ordering.
// Serving processes that pin every byte of HBM to a pool at start-up are in
// the same position.  For them this entry point takes its per-simulation
// buffers from one fixed array compiled into the library instead of a
// caller workspace.
//
// The array is SCACCHI_STATIC_SCRATCH_BYTES (4 MiB) per device.  Every GPU
// on which the library's search module is loaded holds it until the
// process exits, whether or not this entry point is used.

static __device__ __align__(256) uint8_t g_search_scratch[SCACCHI_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxScratchDevices = 64;
// Device address of g_search_scratch per device, resolved on first use in
// the device's current context.  A context torn down and created again
// (cudaDeviceReset, a primary-context reset) reloads the module at a new
// address, so the address is kept together with the context it was
// resolved in and resolved again when the current context differs.
struct ScratchSlot {
  CUcontext ctx = nullptr;
  void *addr = nullptr;
};
ScratchSlot g_scratch_slot[kMaxScratchDevices];
std::mutex g_scratch_mutex;

PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  return fn;
}

}  // namespace

extern "C" {

int scacchi_search_synthetic_static(const scacchi_tree *tree, const scacchi_synthetic_params *env,
                                    const uint32_t *keys, int32_t num_simulations, int32_t max_depth,
                                    const scacchi_update_params *params, uint64_t *stats, void *stream) {
  // the descriptor first (a malformed call is EINVAL whatever its size),
  // then the size against the array
  if (!tree_ok(tree) || !env || !keys || num_simulations < 0 || max_depth < 1 || !params_ok(params) ||
      env->num_actions != tree->num_actions || tree->emb_bytes != (int32_t)sizeof(se_state) ||
      num_simulations + 1 > tree->num_nodes)
    return SCACCHI_EINVAL;
  const size_t need = scacchi_search_workspace_bytes(tree->batch, tree->num_actions, tree->emb_bytes);
  if (need > (size_t)SCACCHI_STATIC_SCRATCH_BYTES) return SCACCHI_ETOOLARGE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return SCACCHI_ECUDA;
  if (dev < 0 || dev >= kMaxScratchDevices) return SCACCHI_ECUDA;
  CUcontext ctx = nullptr;
  auto get_ctx = ctx_get_current();
  if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS) return SCACCHI_ECUDA;
  void *scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchSlot &slot = g_scratch_slot[dev];
    if (!ctx || slot.ctx != ctx || !slot.addr) {
      // Set-up, once per device and context, with that device current
      // (the lookup also makes the runtime create the device's context if
      // this thread has none yet).
      if (cudaGetSymbolAddress(&scratch, g_search_scratch) != cudaSuccess || !scratch) return SCACCHI_ECUDA;
      if (!ctx && (get_ctx(&ctx) != CUDA_SUCCESS || !ctx)) return SCACCHI_ECUDA;
      slot.ctx = ctx;
      slot.addr = scratch;
    }
    scratch = slot.addr;
  }
  // Every scratch byte a simulation reads is written earlier in the same
  // simulation (the descent writes parent, action, active and the parent
  // state of every lane; the game step writes all its outputs), so the
  // previous call's contents need no clearing.
  return scacchi_search_synthetic(tree, env, keys, num_simulations, max_depth, params, scratch, stats, stream);
}

}  // extern "C"
