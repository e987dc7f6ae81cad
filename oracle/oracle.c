/*
 * CPU oracle for the batched Dirichlet-Thompson search step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, lane by lane in plain C, the
 * algorithm of the reference's `scacchi/dirichlet_mctx` package (citations are
 * to files of Francesco215/Scacchi).  It is the checker for the CUDA kernels
 * and the timed CPU baseline; no product code path calls it.
 *
 * Floating point: the oracle and the kernels share two leaf headers, the
 * Threefry/jax.random layer (threefry.h) and the scalar math (smath.h).
 * Reductions over the action axis use one canonical order that the warp
 * kernels also use ("warp order": per slot t < 32 the partial
 * v[t] + v[t+32] + v[t+64] + v[t+96] over present actions, then a butterfly
 * p[t] + p[t^16], ^8, ^4, ^2, ^1).  Sums over the quadrature grid run in
 * increasing grid order.  The reference leaves these orders to XLA.
 *
 * Outcomes are binary (O = 2, loss index 0, win index 1), the Hex case.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../scacchi_b200/csrc/synthetic_env.h"

#define NO_OUTCOME (-1)
#define NO_PARENT (-1)
#define UNVISITED (-1)
#define MAX_ACTIONS 128

/* ------------------------------------------------------------------ */
/* canonical reductions                                                 */
/* ------------------------------------------------------------------ */

static float warp_order_sum(const float *v, int n) {
  float p[32];
  for (int t = 0; t < 32; ++t) {
    float s = 0.0f;
    int first = 1;
    for (int j = t; j < n; j += 32) {
      if (first) {
        s = v[j];
        first = 0;
      } else {
        s = s + v[j];
      }
    }
    p[t] = s;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float q[32];
    for (int t = 0; t < 32; ++t) q[t] = p[t] + p[t ^ off];
    memcpy(p, q, sizeof(p));
  }
  return p[0];
}

/* jnp.argmax: first NaN if any, else first maximum. */
static int nan_first_argmax(const float *v, int n) {
  int best = 0;
  for (int i = 1; i < n; ++i) {
    float a = v[i], b = v[best];
    int better;
    if (sm_isnan(b)) better = 0;
    else if (sm_isnan(a)) better = 1;
    else better = a > b;
    if (better) best = i;
  }
  return best;
}

/* ------------------------------------------------------------------ */
/* outcomes.py                                                          */
/* ------------------------------------------------------------------ */

/* align_categorical_outcome, outcomes.py:21-27 (O = 2) */
static int8_t align_cat(int8_t outcome, int32_t source, int32_t target) {
  if (outcome == NO_OUTCOME) return NO_OUTCOME;
  return source == target ? outcome : (int8_t)(1 - outcome);
}

/* align_outcome, outcomes.py:17-18 */
static void align_alpha(const float *a, int32_t source, int32_t target, float *out) {
  if (source == target) {
    out[0] = a[0];
    out[1] = a[1];
  } else {
    float t0 = a[1], t1 = a[0];
    out[0] = t0;
    out[1] = t1;
  }
}

/* ------------------------------------------------------------------ */
/* action_selection.py                                                  */
/* ------------------------------------------------------------------ */

/* One Gamma log-variate of sample_dirichlet (action_selection.py:100-130)
 * at flat index idx of a [*shape] draw whose proposal axis has stride
 * `stride` (= prod(shape)). */
static float log_gamma_draw(sk_key normal_key, sk_key accept_key, sk_key augment_key,
                            uint64_t idx, uint64_t stride, float alpha_in) {
  float alpha = alpha_in > SM_TINY ? alpha_in : SM_TINY;
  if (sm_isnan(alpha_in)) alpha = alpha_in;
  float shape = alpha < 1.0f ? alpha + 1.0f : alpha;
  float d = shape - 0.333333343f;
  float c = sm_rsqrtf(9.0f * d);
  float chosen = 0.0f;
  int found = 0;
  float z0 = 0.0f;
  for (int p = 0; p < 4; ++p) {
    uint64_t i = (uint64_t)p * stride + idx;
    float z = sk_normal(normal_key, i);
    if (p == 0) z0 = z;
    float base = 1.0f + c * z;
    if (!(base > 0.0f)) continue;
    float cube = base * (base * base);
    float u = sk_uniform_tiny(accept_key, i);
    float z2 = z * z;
    int accept = u < 1.0f - 0.0331f * (z2 * z2);
    if (!accept) accept = sm_logf(u) < 0.5f * z2 + d * ((1.0f - cube) + sm_logf(cube));
    if (accept) {
      chosen = cube;
      found = 1;
      break;
    }
  }
  if (!found) {
    float fb = 1.0f + c * z0;
    float floor_ = sqrtf(SM_TINY);
    fb = fb > floor_ ? fb : floor_;
    chosen = fb * (fb * fb);
  }
  float lg = sm_logf(d) + sm_logf(chosen);
  if (alpha < 1.0f) {
    float u = sk_uniform_tiny(augment_key, idx);
    lg = lg + sm_logf(u) / alpha;
  }
  return lg;
}

/* outcome_utility(softmax(log_gamma)) for O = 2 (action_selection.py:132,
 * outcomes.py:34-35) */
static float binary_utility(float lg0, float lg1) {
  float m = lg0 > lg1 ? lg0 : lg1;
  if (sm_isnan(lg0) || sm_isnan(lg1)) m = SM_NAN;
  float e0 = sm_expf(lg0 - m);
  float e1 = sm_expf(lg1 - m);
  float s = e0 + e1;
  return e1 / s - e0 / s;
}

/* thompson_sample (action_selection.py:135-143) for lane `b` of a batched
 * [B, A, 2] draw.  `masked` is the argmax mask; `cat` (or NULL) overrides the
 * sampled utility with the exact categorical utility. */
static int thompson_lane(sk_key key, const float *alpha, const uint8_t *masked,
                         const int8_t *cat, int A, int b, int B) {
  sk_key proposal = sk_split(key, 0), augment = sk_split(key, 1);
  sk_key normal_key = sk_split(proposal, 0), accept_key = sk_split(proposal, 1);
  uint64_t stride = (uint64_t)B * (uint64_t)A * 2u;
  float util[MAX_ACTIONS];
  for (int a = 0; a < A; ++a) {
    if (masked[a]) {
      util[a] = -SM_INF;
      continue;
    }
    if (cat && cat[a] != NO_OUTCOME) {
      util[a] = cat[a] == 1 ? 1.0f : (cat[a] == 0 ? -1.0f : 0.0f);
      continue;
    }
    uint64_t base = (uint64_t)b * (uint64_t)A * 2u + (uint64_t)a * 2u;
    float lg0 = log_gamma_draw(normal_key, accept_key, augment, base, stride, alpha[2 * a]);
    float lg1 = log_gamma_draw(normal_key, accept_key, augment, base + 1, stride, alpha[2 * a + 1]);
    util[a] = binary_utility(lg0, lg1);
  }
  return nan_first_argmax(util, A);
}

/* posterior_best_policy (action_selection.py:146-194) for lane b of B. */
static void posterior_best_policy_lane(sk_key key, const float *alpha, const uint8_t *invalid,
                                       const int8_t *cat, int A, int S, int b, int B,
                                       float *policy) {
  if (S == 1) {
    int best = thompson_lane(key, alpha, invalid, cat, A, b, B);
    for (int a = 0; a < A; ++a) policy[a] = (!invalid[a] && a == best) ? 1.0f : 0.0f;
    return;
  }
  sk_key sample_key = sk_split(key, 0);
  float hits[MAX_ACTIONS];
  for (int a = 0; a < A; ++a) hits[a] = 0.0f;
  for (int s = 0; s < S; ++s) {
    int best = thompson_lane(sk_split(sample_key, (uint64_t)s), alpha, invalid, cat, A, b, B);
    hits[best] = hits[best] + 1.0f;
  }
  float fS = (float)S;
  int legal_count = 0;
  for (int a = 0; a < A; ++a) {
    policy[a] = invalid[a] ? 0.0f : hits[a] / fS;
    legal_count += !invalid[a];
  }
  float total = warp_order_sum(policy, A);
  float denom = total > 1.0f ? total : 1.0f;
  float lc = (float)(legal_count > 1 ? legal_count : 1);
  for (int a = 0; a < A; ++a) {
    if (total > 0.0f) policy[a] = policy[a] / denom;
    else policy[a] = (invalid[a] ? 0.0f : 1.0f) / lc;
  }
}

/* _categorical_candidates (action_selection.py:24-49), O = 2 */
static int categorical_candidates(int8_t node_outcome, const int8_t *edge_outcome,
                                  const int32_t *edge_distance, const uint8_t *invalid, int A,
                                  uint8_t *tied) {
  float scores[MAX_ACTIONS];
  float best = -SM_INF;
  for (int a = 0; a < A; ++a) {
    int legal = !invalid[a];
    float dist = (float)edge_distance[a];
    float s;
    if (node_outcome == 1) s = (legal && edge_outcome[a] == 1) ? -dist : -SM_INF;
    else if (node_outcome == 0) s = (legal && edge_outcome[a] == 0) ? dist : -SM_INF;
    else s = (legal && edge_outcome[a] == 1) ? 0.0f : -SM_INF;
    scores[a] = s;
    if (s > best) best = s;
  }
  int count = 0;
  for (int a = 0; a < A; ++a) {
    tied[a] = sm_isfinite(scores[a]) && scores[a] == best;
    count += tied[a];
  }
  return count;
}

/* ------------------------------------------------------------------ */
/* prefix_cdf.py                                                        */
/* ------------------------------------------------------------------ */

typedef struct {
  int half_width;
  float tail_scale;
  float min_half_range;
  float max_half_range;
} or_prefix_params;

typedef struct {
  float *policy;          /* [A] */
  float *raw_policy;      /* [A] */
  float *raw_mass;        /* [1] */
  float *normalization_error;
  uint8_t *finite;
  float *grid_half_range;
  uint8_t *tail_range_clipped;
  float *density_log_integral; /* [A] */
  int32_t *fallback_interval_count;
} or_prefix_out;

static float log_cosh(float v) {
  float a = v < 0.0f ? -v : v;
  return (a + sm_log1pf(sm_expf(-2.0f * a))) - sm_logf(2.0f);
}

/* binary_posterior_best_policy_prefix_quadrature, prefix_cdf.py:217-445,
 * one lane. */
static void prefix_cdf_lane(const float *alpha, const uint8_t *invalid, const int8_t *outcome,
                            int A, const or_prefix_params *prm, or_prefix_out *o, int lane) {
  const int h = prm->half_width;
  const int Q = 2 * h + 1;
  uint8_t unres[MAX_ACTIONS], legal[MAX_ACTIONS], cwin[MAX_ACTIONS];
  int has_unres = 0, has_legal = 0, has_cw = 0, n_unres = 0;
  for (int a = 0; a < A; ++a) {
    legal[a] = !invalid[a];
    unres[a] = legal[a] && outcome[a] == NO_OUTCOME;
    cwin[a] = legal[a] && outcome[a] == 1;
    has_unres |= unres[a];
    has_legal |= legal[a];
    has_cw |= cwin[a];
    n_unres += unres[a];
  }
  /* _adaptive_grid_half_range, prefix_cdf.py:68-118 */
  float min_alpha = SM_INF;
  for (int a = 0; a < A; ++a) {
    if (!unres[a]) continue;
    for (int k = 0; k < 2; ++k) {
      float v = alpha[2 * a + k] > SM_TINY ? alpha[2 * a + k] : SM_TINY;
      if (v < min_alpha) min_alpha = v;
    }
  }
  float requested = sm_asinhf_pos(prm->tail_scale / min_alpha);
  if (!has_unres) requested = prm->min_half_range;
  float hr = requested;
  if (hr < prm->min_half_range) hr = prm->min_half_range;
  if (hr > prm->max_half_range) hr = prm->max_half_range;
  int clipped = has_unres && requested > prm->max_half_range;
  float *lx = (float *)malloc(sizeof(float) * Q * 3);
  float *l1mx = lx + Q, *lj = lx + 2 * Q;
  float fh = (float)h;
  for (int k = 0; k < Q; ++k) {
    float unit = (float)(k - h) / fh;
    float coord = hr * unit;
    float logit = sm_sinhf(coord);
    lx[k] = -sm_softplusf(-logit);
    l1mx[k] = -sm_softplusf(logit);
    lj[k] = log_cosh(coord);
  }
  float step = hr / fh;
  float hstep = 0.5f * step;
  /* per action: density, cumulative sums */
  float *dens = (float *)malloc(sizeof(float) * A * Q);
  float *cdf = (float *)malloc(sizeof(float) * A * Q);
  float *flc = (float *)malloc(sizeof(float) * A * Q);
  uint8_t *pos = (uint8_t *)malloc((size_t)A * Q);
  float *nd = (float *)malloc(sizeof(float) * A * Q);
  float dli[MAX_ACTIONS];
  for (int a = 0; a < A; ++a) {
    float w = unres[a] ? (alpha[2 * a + 1] > SM_TINY ? alpha[2 * a + 1] : SM_TINY) : 1.0f;
    float l = unres[a] ? (alpha[2 * a] > SM_TINY ? alpha[2 * a] : SM_TINY) : 1.0f;
    float bl = sm_betalnf(w, l);
    float scale = -SM_INF;
    int any_nan = 0;
    for (int k = 0; k < Q; ++k) {
      float ld = ((w * lx[k] + l * l1mx[k]) - bl) + lj[k];
      dens[a * Q + k] = ld;
      if (sm_isnan(ld)) any_nan = 1;
      if (ld > scale) scale = ld;
    }
    if (any_nan) scale = SM_NAN;
    for (int k = 0; k < Q; ++k) {
      float d = sm_expf(dens[a * Q + k] - scale);
      dens[a * Q + k] = unres[a] ? d : 0.0f;
    }
    float run = 0.0f;
    cdf[a * Q] = 0.0f;
    for (int k = 0; k + 1 < Q; ++k) {
      float inc = hstep * (dens[a * Q + k] + dens[a * Q + k + 1]);
      run = run + inc;
      cdf[a * Q + k + 1] = run;
    }
    float integral = cdf[a * Q + Q - 1];
    dli[a] = unres[a] ? scale + sm_logf(integral) : 0.0f;
    float safe = integral > 0.0f ? integral : 1.0f;
    for (int k = 0; k < Q; ++k) {
      float c = cdf[a * Q + k] / safe;
      cdf[a * Q + k] = c;
      nd[a * Q + k] = dens[a * Q + k] / safe;
      pos[a * Q + k] = c > 0.0f;
      flc[a * Q + k] = c > 0.0f ? sm_logf(c) : 0.0f;
    }
  }
  /* leave-one-out products and joint CDF per grid point */
  float *integrand = (float *)malloc(sizeof(float) * A * Q);
  float *joint = (float *)malloc(sizeof(float) * Q);
  float col[MAX_ACTIONS];
  for (int k = 0; k < Q; ++k) {
    int zero_count = 0;
    for (int a = 0; a < A; ++a) {
      zero_count += unres[a] && !pos[a * Q + k];
      col[a] = unres[a] ? flc[a * Q + k] : 0.0f;
    }
    float flp = warp_order_sum(col, A);
    for (int a = 0; a < A; ++a) {
      int zf = unres[a] && !pos[a * Q + k];
      float olp = (zero_count - zf) > 0 ? -SM_INF : flp - flc[a * Q + k];
      integrand[a * Q + k] = nd[a * Q + k] * sm_expf(olp);
      float m = flc[a * Q + k] < 0.0f ? flc[a * Q + k] : 0.0f;
      col[a] = unres[a] ? (pos[a * Q + k] ? m : -SM_INF) : 0.0f;
    }
    joint[k] = sm_expf(warp_order_sum(col, A));
  }
  /* _maximum_cdf, prefix_cdf.py:186-214 */
  joint[0] = has_unres ? 0.0f : 1.0f;
  joint[Q - 1] = 1.0f;
  for (int k = 1; k < Q; ++k) {
    float prev = joint[k - 1];
    if (sm_isnan(prev) || (!sm_isnan(joint[k]) && prev > joint[k])) joint[k] = prev;
  }
  joint[Q - 1] = 1.0f;
  float prob[MAX_ACTIONS];
  for (int a = 0; a < A; ++a) prob[a] = 0.0f;
  float uniform_den = (float)(n_unres > 1 ? n_unres : 1);
  int fallback_intervals = 0;
  for (int j = 0; j + 1 < Q; ++j) {
    float contrib[MAX_ACTIONS];
    for (int a = 0; a < A; ++a) {
      float c = hstep * (integrand[a * Q + j] + integrand[a * Q + j + 1]);
      contrib[a] = c > 0.0f ? c : (sm_isnan(c) ? c : 0.0f);
    }
    float score = warp_order_sum(contrib, A);
    float jinc = joint[j + 1] - joint[j];
    jinc = jinc > 0.0f ? jinc : (sm_isnan(jinc) ? jinc : 0.0f);
    int sp = score > 0.0f;
    if (!sp && jinc > 0.0f) fallback_intervals += 1;
    for (int a = 0; a < A; ++a) {
      float w = sp ? contrib[a] / score : (unres[a] ? 1.0f : 0.0f) / uniform_den;
      prob[a] = prob[a] + w * jinc;
    }
  }
  /* _finalize_policy, prefix_cdf.py:121-183 */
  int first_cw = 0;
  for (int a = A - 1; a >= 0; --a)
    if (cwin[a]) first_cw = a;
  float cscore[MAX_ACTIONS];
  for (int a = 0; a < A; ++a) cscore[a] = legal[a] ? (float)outcome[a] : -SM_INF;
  int cbest = has_cw ? first_cw : nan_first_argmax(cscore, A);
  float raw[MAX_ACTIONS];
  for (int a = 0; a < A; ++a) {
    float r = (has_cw || !has_unres) ? (a == cbest ? 1.0f : 0.0f) : (unres[a] ? prob[a] : 0.0f);
    raw[a] = legal[a] ? r : 0.0f;
  }
  float mass = warp_order_sum(raw, A);
  float nerr = fabsf(mass - (has_legal ? 1.0f : 0.0f));
  float safe_mass = mass > 0.0f ? mass : 1.0f;
  int finite = sm_isfinite(mass) && sm_isfinite(nerr) && sm_isfinite(hr);
  for (int a = 0; a < A; ++a) {
    float p = raw[a] / safe_mass;
    p = has_legal ? p : 0.0f;
    o->policy[lane * A + a] = p;
    o->raw_policy[lane * A + a] = raw[a];
    o->density_log_integral[lane * A + a] = dli[a];
    finite = finite && sm_isfinite(p) && sm_isfinite(raw[a]);
    if (unres[a] && !sm_isfinite(dli[a])) finite = 0;
  }
  o->raw_mass[lane] = mass;
  o->normalization_error[lane] = nerr;
  o->finite[lane] = (uint8_t)finite;
  o->grid_half_range[lane] = hr;
  o->tail_range_clipped[lane] = (uint8_t)clipped;
  o->fallback_interval_count[lane] = fallback_intervals;
  free(lx);
  free(dens);
  free(cdf);
  free(flc);
  free(pos);
  free(nd);
  free(integrand);
  free(joint);
}

/* ------------------------------------------------------------------ */
/* tree.py / posterior_updates.py / utils.py / search.py                */
/* ------------------------------------------------------------------ */

typedef struct {
  int B, C, A, emb_bytes;
  int32_t *parents;
  int32_t *children;
  int32_t *to_play;
  int8_t *node_outcome;
  int32_t *node_payload;
  int8_t *edge_outcome;
  int32_t *edge_payload;
  float *value_prior;
  float *value_alpha;
  float *edge_alpha;
  uint8_t *invalid;
  uint8_t *embedding;
  /* The tree may hold lanes [lane_offset, lane_offset + B) of a batch of
   * total_batch lanes (0 = B): lane-indexed random streams use the global
   * lane index and batch size, so any lane range reproduces the full run. */
  int lane_offset;
  int total_batch;
} or_tree;

static int glane(const or_tree *t, int b) { return b + t->lane_offset; }
static int gbatch(const or_tree *t) { return t->total_batch > 0 ? t->total_batch : t->B; }

typedef struct {
  int rule;               /* 0: update_posterior (MC), 1: update_posterior_prefix_cdf */
  int kappa_ge_one;       /* kappa >= 1 (decided in double precision) */
  float inv_kappa;        /* float32(1 / kappa) */
  float kappa;            /* float32(kappa) */
  int samples;            /* policy_samples or fallback_policy_samples */
  or_prefix_params prefix;
  float density_tol;
} or_update_params;

#define NODE(t, b, n) ((size_t)(b) * (t)->C + (n))
#define EDGE(t, b, n, a) (NODE(t, b, n) * (t)->A + (a))

/* instantiate_tree_from_root, tree.py:245-277 */
void or_tree_init(or_tree *t, const float *root_value, const float *root_action_values,
                  const uint8_t *root_invalid, const int8_t *root_terminal,
                  const int32_t *root_to_play, const uint8_t *root_embedding) {
  for (int b = 0; b < t->B; ++b) {
    for (int n = 0; n < t->C; ++n) {
      size_t i = NODE(t, b, n);
      int root = n == 0;
      t->parents[i] = NO_PARENT;
      t->to_play[i] = root ? root_to_play[b] : 0;
      t->node_outcome[i] = root ? root_terminal[b] : NO_OUTCOME;
      t->node_payload[i] = 0;
      for (int k = 0; k < 2; ++k) {
        float v = root ? root_value[2 * b + k] : 1.0f;
        t->value_prior[2 * i + k] = v;
        t->value_alpha[2 * i + k] = v;
      }
      for (int a = 0; a < t->A; ++a) {
        size_t e = EDGE(t, b, n, a);
        t->children[e] = UNVISITED;
        t->edge_outcome[e] = NO_OUTCOME;
        t->edge_payload[e] = 0;
        t->invalid[e] = root ? root_invalid[b * t->A + a] : 1;
        for (int k = 0; k < 2; ++k)
          t->edge_alpha[2 * e + k] = root ? root_action_values[((size_t)b * t->A + a) * 2 + k] : 1.0f;
      }
      if (t->emb_bytes) {
        uint8_t *dst = t->embedding + i * t->emb_bytes;
        if (root && root_embedding) memcpy(dst, root_embedding + (size_t)b * t->emb_bytes, t->emb_bytes);
        else memset(dst, 0, t->emb_bytes);
      }
    }
  }
}

static int any_searchable(const or_tree *t, int b, int n) {
  for (int a = 0; a < t->A; ++a) {
    size_t e = EDGE(t, b, n, a);
    if (!t->invalid[e] && t->edge_outcome[e] == NO_OUTCOME) return 1;
  }
  return 0;
}

/* effective_action_alpha, action_selection.py:197-215 */
static void effective_alpha_node(const or_tree *t, int b, int n, float *out) {
  int32_t player = t->to_play[NODE(t, b, n)];
  for (int a = 0; a < t->A; ++a) {
    size_t e = EDGE(t, b, n, a);
    int32_t child = t->children[e];
    int visited = child != UNVISITED;
    int use_child = visited && t->edge_outcome[e] == NO_OUTCOME && t->edge_payload[e] <= 0;
    if (use_child) {
      size_t ci = NODE(t, b, child);
      align_alpha(t->value_prior + 2 * ci, t->to_play[ci], player, out + 2 * a);
    } else {
      out[2 * a] = t->edge_alpha[2 * e];
      out[2 * a + 1] = t->edge_alpha[2 * e + 1];
    }
  }
}

/* _simulate_one / simulate, search.py:21-78 */
void or_simulate(const or_tree *t, sk_key simulate_key, int max_depth, int32_t *parent_out,
                 int32_t *action_out, uint8_t *active_out) {
  float alpha[2 * MAX_ACTIONS];
  uint8_t masked[MAX_ACTIONS];
  for (int b = 0; b < t->B; ++b) {
    sk_key key = sk_split(simulate_key, (uint64_t)glane(t, b));
    int root_active = t->node_outcome[NODE(t, b, 0)] == NO_OUTCOME && any_searchable(t, b, 0);
    int node = 0, next = 0, action = 0, depth = 0, cont = root_active;
    while (cont) {
      sk_key next_key = sk_split(key, 0), sel_key = sk_split(key, 1);
      node = next;
      effective_alpha_node(t, b, node, alpha);
      for (int a = 0; a < t->A; ++a) {
        size_t e = EDGE(t, b, node, a);
        masked[a] = t->invalid[e] || t->edge_outcome[e] != NO_OUTCOME;
      }
      action = thompson_lane(sel_key, alpha, masked, NULL, t->A, 0, 1);
      int32_t child = t->children[EDGE(t, b, node, action)];
      int visited = child != UNVISITED;
      int safe = visited ? child : 0;
      depth += 1;
      int selectable = t->node_outcome[NODE(t, b, safe)] == NO_OUTCOME && any_searchable(t, b, safe);
      cont = visited && selectable && depth < max_depth;
      next = child;
      key = next_key;
    }
    parent_out[b] = node;
    action_out[b] = action;
    active_out[b] = (uint8_t)root_active;
  }
}

/* expand, search.py:101-143 (recurrent outputs supplied by the caller) */
void or_expand(or_tree *t, int new_node, const int32_t *sim_parent, const int32_t *sim_action,
               const uint8_t *sim_active, const float *step_value, const float *step_action_values,
               const uint8_t *step_invalid, const int8_t *step_terminal, const int32_t *step_to_play,
               const uint8_t *step_embedding) {
  for (int b = 0; b < t->B; ++b) {
    int active = sim_active[b];
    int parent = active ? sim_parent[b] : 0;
    int action = active ? sim_action[b] : 0;
    size_t pe = EDGE(t, b, parent, action);
    size_t pn = NODE(t, b, parent);
    int32_t child = t->children[pe];
    int initialize = active && child == UNVISITED;
    int8_t outcome = step_terminal[b];
    int8_t aligned = align_cat(outcome, step_to_play[b], t->to_play[pn]);
    int publish = active && outcome != NO_OUTCOME;
    int32_t old_count = t->edge_payload[pe];
    int32_t parent_support = t->node_payload[pn] + (1 - old_count);
    if (initialize && new_node >= 0 && new_node < t->C) {
      size_t ni = NODE(t, b, new_node);
      t->parents[ni] = parent;
      t->children[pe] = new_node;
      t->to_play[ni] = step_to_play[b];
      t->node_outcome[ni] = outcome;
      for (int k = 0; k < 2; ++k) {
        t->value_prior[2 * ni + k] = step_value[2 * b + k];
        t->value_alpha[2 * ni + k] = step_value[2 * b + k];
      }
      for (int a = 0; a < t->A; ++a) {
        size_t e = EDGE(t, b, new_node, a);
        t->invalid[e] = step_invalid[(size_t)b * t->A + a];
        for (int k = 0; k < 2; ++k)
          t->edge_alpha[2 * e + k] = step_action_values[((size_t)b * t->A + a) * 2 + k];
      }
      if (t->emb_bytes && step_embedding)
        memcpy(t->embedding + ni * t->emb_bytes, step_embedding + (size_t)b * t->emb_bytes, t->emb_bytes);
    }
    if (publish) {
      t->node_payload[pn] = parent_support;
      t->edge_outcome[pe] = aligned;
      t->edge_payload[pe] = 1;
    }
  }
}

/* mix_value_prior, posterior_updates.py:40-63 */
static void mix_value_prior(const float *prior, const float *cache, const float *policy, int A,
                            int32_t n_down, const or_update_params *u, float *out) {
  float col[MAX_ACTIONS];
  float weighted[2];
  for (int k = 0; k < 2; ++k) {
    for (int a = 0; a < A; ++a) col[a] = policy[a] * cache[2 * a + k];
    weighted[k] = warp_order_sum(col, A);
  }
  float n = (float)n_down;
  float pw, dw;
  if (u->kappa_ge_one) {
    float rc = n * u->inv_kappa;
    float den = 1.0f + rc;
    pw = 1.0f / den;
    dw = rc / den;
  } else {
    float den = u->kappa + n;
    pw = u->kappa / den;
    dw = n / den;
  }
  for (int k = 0; k < 2; ++k) out[k] = pw * prior[k] + dw * weighted[k];
}

/* One posterior update context, gathered as in utils.py:35-50. */
typedef struct {
  int active;
  int leaf_active;
  int32_t leaf_action;
  float leaf_value[2];
  int32_t leaf_to_play;
  int32_t node_to_play;
  int32_t node_payload;
  float value_prior[2];
  float value_alpha[2];
  float edge_alpha[2 * MAX_ACTIONS];
  int32_t edge_payload[MAX_ACTIONS];
  int8_t edge_outcome[MAX_ACTIONS];
  uint8_t invalid[MAX_ACTIONS];
  uint8_t child_visited[MAX_ACTIONS];
  float child_prior[2 * MAX_ACTIONS];
  float child_value[2 * MAX_ACTIONS];
  int32_t child_payload[MAX_ACTIONS];
  int8_t child_outcome[MAX_ACTIONS];
  int32_t child_to_play[MAX_ACTIONS];
} or_context;

typedef struct {
  float edge_alpha[2 * MAX_ACTIONS];
  int32_t edge_payload[MAX_ACTIONS];
  float value_alpha[2];
  uint8_t unsafe;  /* prefix-CDF lane sent to the MC fallback */
} or_update;

/* _repair_inputs + the rule + _repair_from_policy,
 * posterior_updates.py:66-367, for lane b of B. */
static void posterior_update_lane(sk_key update_key, const or_context *c, int A,
                                  const or_update_params *u, int b, int B, or_update *out) {
  float eff[2 * MAX_ACTIONS] = {0}, cache[2 * MAX_ACTIONS] = {0};
  int32_t count_delta = 0;
  int leaf_action = c->leaf_action < 0 ? c->leaf_action + A : c->leaf_action;
  float direct[2];
  align_alpha(c->leaf_value, c->leaf_to_play, c->node_to_play, direct);
  for (int a = 0; a < A; ++a) {
    int unresolved = c->edge_outcome[a] == NO_OUTCOME;
    float ea0 = c->edge_alpha[2 * a], ea1 = c->edge_alpha[2 * a + 1];
    int32_t ep = c->edge_payload[a];
    if (c->leaf_active && a == leaf_action && unresolved) {
      ea0 = direct[0];
      ea1 = direct[1];
      ep = ep + 1;
    }
    int refresh = c->active && c->child_visited[a] && c->child_outcome[a] == NO_OUTCOME &&
                  c->child_payload[a] > 0 && unresolved;
    if (refresh) {
      float cv[2];
      align_alpha(c->child_value + 2 * a, c->child_to_play[a], c->node_to_play, cv);
      ea0 = cv[0];
      ea1 = cv[1];
      ep = 1 + c->child_payload[a];
    }
    out->edge_alpha[2 * a] = ea0;
    out->edge_alpha[2 * a + 1] = ea1;
    out->edge_payload[a] = ep;
    int use_child_prior = c->child_visited[a] && unresolved && ep <= 0;
    if (use_child_prior) {
      align_alpha(c->child_prior + 2 * a, c->child_to_play[a], c->node_to_play, eff + 2 * a);
    } else {
      eff[2 * a] = ea0;
      eff[2 * a + 1] = ea1;
    }
    if (!unresolved) {
      /* sum(alpha) * one_hot(outcome), posterior_updates.py:153-174 */
      float s = eff[2 * a] + eff[2 * a + 1];
      int oc = c->edge_outcome[a];
      cache[2 * a] = s * (oc == 0 ? 1.0f : 0.0f);
      cache[2 * a + 1] = s * (oc == 1 ? 1.0f : 0.0f);
    } else {
      cache[2 * a] = eff[2 * a];
      cache[2 * a + 1] = eff[2 * a + 1];
    }
    if (unresolved && !c->invalid[a]) count_delta += ep - c->edge_payload[a];
  }
  int32_t n_down = c->node_payload + count_delta;
  float policy[MAX_ACTIONS];
  out->unsafe = 0;
  if (u->rule == 1) {
    float raw[MAX_ACTIONS], dli[MAX_ACTIONS], mass, nerr, hr;
    uint8_t finite, clipped;
    int32_t fic;
    or_prefix_out po = {policy, raw, &mass, &nerr, &finite, &hr, &clipped, dli, &fic};
    prefix_cdf_lane(eff, c->invalid, c->edge_outcome, A, &u->prefix, &po, 0);
    float derr = 0.0f;
    int derr_nan = 0;
    for (int a = 0; a < A; ++a) {
      float v = fabsf(dli[a]);
      if (sm_isnan(v)) derr_nan = 1;
      if (v > derr) derr = v;
    }
    int too_large = !derr_nan && derr > u->density_tol;
    int unsafe = c->active && (clipped || !finite || too_large);
    if (unsafe) {
      out->unsafe = 1;
      posterior_best_policy_lane(update_key, eff, c->invalid, c->edge_outcome, A, u->samples, b, B, policy);
    }
  } else {
    posterior_best_policy_lane(update_key, eff, c->invalid, c->edge_outcome, A, u->samples, b, B, policy);
  }
  float repaired[2];
  mix_value_prior(c->value_prior, cache, policy, A, n_down, u, repaired);
  if (c->active && n_down > 0) {
    out->value_alpha[0] = repaired[0];
    out->value_alpha[1] = repaired[1];
  } else {
    out->value_alpha[0] = c->value_alpha[0];
    out->value_alpha[1] = c->value_alpha[1];
  }
}

/* _gather_node / _gather_children, utils.py:35-50 */
static void gather_context(const or_tree *t, int b, int n, int active, int leaf_active,
                           int32_t leaf_action, const float *leaf_value, int32_t leaf_to_play,
                           or_context *c) {
  size_t ni = NODE(t, b, n);
  c->active = active;
  c->leaf_active = leaf_active;
  c->leaf_action = leaf_action;
  c->leaf_value[0] = leaf_value[0];
  c->leaf_value[1] = leaf_value[1];
  c->leaf_to_play = leaf_to_play;
  c->node_to_play = t->to_play[ni];
  c->node_payload = t->node_payload[ni];
  for (int k = 0; k < 2; ++k) {
    c->value_prior[k] = t->value_prior[2 * ni + k];
    c->value_alpha[k] = t->value_alpha[2 * ni + k];
  }
  for (int a = 0; a < t->A; ++a) {
    size_t e = EDGE(t, b, n, a);
    c->edge_alpha[2 * a] = t->edge_alpha[2 * e];
    c->edge_alpha[2 * a + 1] = t->edge_alpha[2 * e + 1];
    c->edge_payload[a] = t->edge_payload[e];
    c->edge_outcome[a] = t->edge_outcome[e];
    c->invalid[a] = t->invalid[e];
    int32_t child = t->children[e];
    c->child_visited[a] = child != UNVISITED;
    size_t ci = NODE(t, b, child != UNVISITED ? child : 0);
    for (int k = 0; k < 2; ++k) {
      c->child_prior[2 * a + k] = t->value_prior[2 * ci + k];
      c->child_value[2 * a + k] = t->value_alpha[2 * ci + k];
    }
    c->child_payload[a] = t->node_payload[ci];
    c->child_outcome[a] = t->node_outcome[ci];
    c->child_to_play[a] = t->to_play[ci];
  }
}

/* _set_node_update, utils.py:53-64 */
static void set_node_update(or_tree *t, int b, int n, const or_update *u) {
  size_t ni = NODE(t, b, n);
  int32_t delta = 0;
  for (int a = 0; a < t->A; ++a) {
    size_t e = EDGE(t, b, n, a);
    if (t->edge_outcome[e] != NO_OUTCOME) continue;
    if (!t->invalid[e]) delta += u->edge_payload[a] - t->edge_payload[e];
    t->edge_payload[e] = u->edge_payload[a];
    t->edge_alpha[2 * e] = u->edge_alpha[2 * a];
    t->edge_alpha[2 * e + 1] = u->edge_alpha[2 * a + 1];
  }
  t->node_payload[ni] += delta;
  t->value_alpha[2 * ni] = u->value_alpha[0];
  t->value_alpha[2 * ni + 1] = u->value_alpha[1];
}

/* _categorize_node_and_publish, utils.py:67-124 (O = 2) */
static void categorize_and_publish(or_tree *t, int b, int n) {
  size_t ni = NODE(t, b, n);
  int has_legal = 0, all_cat = 1, has_win = 0;
  int32_t shortest_win = INT32_MAX, longest_loss = INT32_MIN;
  for (int a = 0; a < t->A; ++a) {
    size_t e = EDGE(t, b, n, a);
    int legal = !t->invalid[e];
    int known = legal && t->edge_outcome[e] != NO_OUTCOME;
    has_legal |= legal;
    if (legal && !known) all_cat = 0;
    if (known && t->edge_outcome[e] == 1) {
      has_win = 1;
      if (t->edge_payload[e] < shortest_win) shortest_win = t->edge_payload[e];
    }
    if (known && t->edge_outcome[e] == 0 && t->edge_payload[e] > longest_loss)
      longest_loss = t->edge_payload[e];
  }
  all_cat = all_cat && has_legal;
  int8_t candidate = has_win ? 1 : (all_cat ? 0 : NO_OUTCOME);
  int32_t cdist = has_win ? shortest_win : longest_loss;
  int8_t old_outcome = t->node_outcome[ni];
  int32_t old_support = t->node_payload[ni];
  int publish_node = old_outcome == NO_OUTCOME && candidate != NO_OUTCOME;
  int32_t parent = t->parents[ni];
  int has_parent = parent != NO_PARENT;
  int safe_parent = has_parent ? parent : 0;
  int incoming_action = 0, has_incoming = 0;
  for (int a = 0; a < t->A; ++a) {
    if (t->children[EDGE(t, b, safe_parent, a)] == n) {
      incoming_action = a;
      has_incoming = 1;
      break;
    }
  }
  size_t pe = EDGE(t, b, safe_parent, incoming_action);
  size_t pn = NODE(t, b, safe_parent);
  int publish_edge = publish_node && has_parent && has_incoming && t->edge_outcome[pe] == NO_OUTCOME;
  int32_t new_parent_support = t->node_payload[pn] + 1 + old_support - t->edge_payload[pe];
  int8_t aligned = align_cat(candidate, t->to_play[ni], t->to_play[pn]);
  if (publish_edge) t->node_payload[pn] = new_parent_support;
  if (publish_node) {
    t->node_payload[ni] = cdist;
    t->node_outcome[ni] = candidate;
  }
  if (publish_edge) {
    t->edge_outcome[pe] = aligned;
    t->edge_payload[pe] = cdist + 1;
  }
}

/* backward, search.py:146-171.  Returns the number of unsafe (fallback)
 * prefix-CDF node updates. */
long or_backward(or_tree *t, sk_key backward_key, const int32_t *sim_parent, const int32_t *sim_action,
                 const uint8_t *sim_active, const float *step_value, const int32_t *step_to_play,
                 const or_update_params *u) {
  long unsafe_count = 0;
  or_context *ctx = (or_context *)malloc(sizeof(or_context));
  or_update *upd = (or_update *)malloc(sizeof(or_update));
  for (int b = 0; b < t->B; ++b) {
    int active = sim_active[b];
    int node = active ? sim_parent[b] : 0;
    int leaf_active = active;
    sk_key key = backward_key;
    while (active) {
      sk_key next_key = sk_split(key, 0), update_key = sk_split(key, 1);
      gather_context(t, b, node, active, leaf_active, sim_action[b], step_value + 2 * b, step_to_play[b], ctx);
      posterior_update_lane(update_key, ctx, t->A, u, glane(t, b), gbatch(t), upd);
      unsafe_count += upd->unsafe;
      set_node_update(t, b, node, upd);
      categorize_and_publish(t, b, node);
      int up = node != 0;
      int parent = t->parents[NODE(t, b, node)];
      node = up ? parent : 0;
      active = up;
      leaf_active = 0;
      key = next_key;
    }
  }
  free(ctx);
  free(upd);
  return unsafe_count;
}

/* tree.summary(), tree.py:212-242 */
void or_summary(const or_tree *t, float *visit_counts, float *alpha, float *value_alpha,
                int8_t *q_outcome, int32_t *q_distance, int8_t *v_outcome, int32_t *v_distance) {
  for (int b = 0; b < t->B; ++b) {
    size_t ri = NODE(t, b, 0);
    effective_alpha_node(t, b, 0, alpha + (size_t)b * t->A * 2);
    for (int a = 0; a < t->A; ++a) {
      size_t e = EDGE(t, b, 0, a);
      int unresolved = t->edge_outcome[e] == NO_OUTCOME;
      visit_counts[(size_t)b * t->A + a] = unresolved ? (float)t->edge_payload[e] : 0.0f;
      q_outcome[(size_t)b * t->A + a] = t->edge_outcome[e];
      q_distance[(size_t)b * t->A + a] = unresolved ? -1 : t->edge_payload[e];
    }
    value_alpha[2 * b] = t->value_alpha[2 * ri];
    value_alpha[2 * b + 1] = t->value_alpha[2 * ri + 1];
    v_outcome[b] = t->node_outcome[ri];
    v_distance[b] = t->node_outcome[ri] == NO_OUTCOME ? -1 : t->node_payload[ri];
  }
}

/* dirichlet_thompson_policy root readout, policies.py:28-42: categorical
 * root one-hot or the posterior-best population, then masked_argmax. */
void or_root_policy(const or_tree *t, sk_key policy_key, const uint8_t *invalid, int samples,
                    float *weights, int32_t *action) {
  const int A = t->A;
  float alpha[2 * MAX_ACTIONS];
  uint8_t tied[MAX_ACTIONS];
  float noise[MAX_ACTIONS];
  sk_key tie_key = sk_fold_in(policy_key, 0);
  int S = samples > 1 ? samples : 1;
  for (int b = 0; b < t->B; ++b) {
    size_t ri = NODE(t, b, 0);
    const uint8_t *inv = invalid + (size_t)b * A;
    float *w = weights + (size_t)b * A;
    if (t->node_outcome[ri] != NO_OUTCOME) {
      /* categorical_action with jax.random.categorical = argmax(gumbel + logits) */
      int count = categorical_candidates(t->node_outcome[ri], t->edge_outcome + EDGE(t, b, 0, 0),
                                         t->edge_payload + EDGE(t, b, 0, 0), inv, A, tied);
      for (int a = 0; a < A; ++a) {
        float u = sk_uniform_tiny(tie_key, (uint64_t)glane(t, b) * A + a);
        float g = -sm_logf(-sm_logf(u));
        noise[a] = g + (tied[a] ? 0.0f : -SM_INF);
      }
      int chosen = count > 0 ? nan_first_argmax(noise, A) : 0;
      for (int a = 0; a < A; ++a) w[a] = a == chosen ? 1.0f : 0.0f;
    } else {
      effective_alpha_node(t, b, 0, alpha);
      posterior_best_policy_lane(policy_key, alpha, inv, t->edge_outcome + EDGE(t, b, 0, 0), A, S, glane(t, b),
                                 gbatch(t), w);
    }
    float masked[MAX_ACTIONS];
    for (int a = 0; a < A; ++a) masked[a] = inv[a] ? -SM_INF : w[a];
    action[b] = nan_first_argmax(masked, A);
  }
}

/* ------------------------------------------------------------------ */
/* unit entry points used by the tests                                  */
/* ------------------------------------------------------------------ */

void or_prefix_cdf(const float *alpha, const uint8_t *invalid, const int8_t *outcome, int B, int A,
                   const or_prefix_params *p, or_prefix_out *o) {
  for (int b = 0; b < B; ++b)
    prefix_cdf_lane(alpha + (size_t)b * A * 2, invalid + (size_t)b * A, outcome + (size_t)b * A, A, p, o,
                    b);
}

void or_posterior_best_policy(sk_key key, const float *alpha, const uint8_t *invalid, const int8_t *cat,
                              int B, int A, int S, float *policy) {
  for (int b = 0; b < B; ++b)
    posterior_best_policy_lane(key, alpha + (size_t)b * A * 2, invalid + (size_t)b * A,
                               cat ? cat + (size_t)b * A : NULL, A, S, b, B, policy + (size_t)b * A);
}

void or_thompson_sample(sk_key key, const float *alpha, const uint8_t *invalid, const int8_t *cat, int B,
                        int A, int32_t *out) {
  for (int b = 0; b < B; ++b)
    out[b] = thompson_lane(key, alpha + (size_t)b * A * 2, invalid + (size_t)b * A,
                           cat ? cat + (size_t)b * A : NULL, A, b, B);
}

/* sample_dirichlet(key, alpha[n, 2]) -> simplex[n, 2] */
void or_sample_dirichlet(sk_key key, const float *alpha, int n, float *out) {
  sk_key proposal = sk_split(key, 0), augment = sk_split(key, 1);
  sk_key normal_key = sk_split(proposal, 0), accept_key = sk_split(proposal, 1);
  uint64_t stride = (uint64_t)n * 2u;
  for (int i = 0; i < n; ++i) {
    float lg0 = log_gamma_draw(normal_key, accept_key, augment, 2u * i, stride, alpha[2 * i]);
    float lg1 = log_gamma_draw(normal_key, accept_key, augment, 2u * i + 1, stride, alpha[2 * i + 1]);
    float m = lg0 > lg1 ? lg0 : lg1;
    float e0 = sm_expf(lg0 - m), e1 = sm_expf(lg1 - m);
    float s = e0 + e1;
    out[2 * i] = e0 / s;
    out[2 * i + 1] = e1 / s;
  }
}

/* update_posterior[_prefix_cdf] on explicit contexts (arrays of B). */
void or_update_posterior(sk_key key, const or_context *ctx, int B, int A, const or_update_params *u,
                         or_update *out) {
  for (int b = 0; b < B; ++b) posterior_update_lane(key, ctx + b, A, u, b, B, out + b);
}

size_t or_sizeof_context(void) { return sizeof(or_context); }
size_t or_sizeof_update(void) { return sizeof(or_update); }

/* ------------------------------------------------------------------ */
/* jax.random primitives exposed for the known-answer tests             */
/* ------------------------------------------------------------------ */

void or_threefry(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t *out) {
  sk_key k = {k0, k1};
  sk_key r = sk_threefry(k, c0, c1);
  out[0] = r.k0;
  out[1] = r.k1;
}

void or_random_bits(uint32_t k0, uint32_t k1, uint64_t n, uint32_t *out) {
  sk_key k = {k0, k1};
  for (uint64_t i = 0; i < n; ++i) out[i] = sk_bits(k, i);
}

void or_uniform(uint32_t k0, uint32_t k1, uint64_t n, float lo, float hi, float *out) {
  sk_key k = {k0, k1};
  for (uint64_t i = 0; i < n; ++i) out[i] = sk_uniform(k, i, lo, hi);
}

void or_normal(uint32_t k0, uint32_t k1, uint64_t n, float *out) {
  sk_key k = {k0, k1};
  for (uint64_t i = 0; i < n; ++i) out[i] = sk_normal(k, i);
}

/* scalar math, vectorised for tests/test_oracle_pins.py */
void or_math(int fn, const float *x, const float *y, int n, float *out) {
  for (int i = 0; i < n; ++i) {
    float v = x[i];
    switch (fn) {
      case 0: out[i] = sm_logf(v); break;
      case 1: out[i] = sm_expf(v); break;
      case 2: out[i] = sm_log1pf(v); break;
      case 3: out[i] = sm_expm1f(v); break;
      case 4: out[i] = sm_lgammaf(v); break;
      case 5: out[i] = sm_betalnf(v, y[i]); break;
      case 6: out[i] = sm_erfinvf(v); break;
      case 7: out[i] = sm_sinhf(v); break;
      case 8: out[i] = sm_asinhf_pos(v); break;
      case 9: out[i] = sm_softplusf(v); break;
      default: out[i] = SM_NAN;
    }
  }
}

/* ------------------------------------------------------------------ */
/* explicit update contexts (struct of arrays), for repair unit tests   */
/* ------------------------------------------------------------------ */

typedef struct {
  const uint8_t *active;        /* [B] */
  const uint8_t *leaf_active;   /* [B] */
  const int32_t *leaf_action;   /* [B] */
  const float *leaf_value;      /* [B,2] */
  const int32_t *leaf_to_play;  /* [B] */
  const int32_t *node_to_play;  /* [B] */
  const int32_t *node_payload;  /* [B] */
  const float *value_prior;     /* [B,2] */
  const float *value_alpha;     /* [B,2] */
  const float *edge_alpha;      /* [B,A,2] */
  const int32_t *edge_payload;  /* [B,A] */
  const int8_t *edge_outcome;   /* [B,A] */
  const uint8_t *invalid;       /* [B,A] */
  const uint8_t *child_visited; /* [B,A] */
  const float *child_prior;     /* [B,A,2] */
  const float *child_value;     /* [B,A,2] */
  const int32_t *child_payload; /* [B,A] */
  const int8_t *child_outcome;  /* [B,A] */
  const int32_t *child_to_play; /* [B,A] */
} or_context_soa;

void or_update_posterior_soa(uint32_t k0, uint32_t k1, const or_context_soa *s, int B, int A,
                             const or_update_params *u, float *out_edge_alpha, int32_t *out_edge_payload,
                             float *out_value_alpha, uint8_t *out_unsafe) {
  sk_key key = {k0, k1};
  or_context *c = (or_context *)malloc(sizeof(or_context));
  or_update *o = (or_update *)malloc(sizeof(or_update));
  for (int b = 0; b < B; ++b) {
    c->active = s->active[b];
    c->leaf_active = s->leaf_active[b];
    c->leaf_action = s->leaf_action[b];
    c->leaf_value[0] = s->leaf_value[2 * b];
    c->leaf_value[1] = s->leaf_value[2 * b + 1];
    c->leaf_to_play = s->leaf_to_play[b];
    c->node_to_play = s->node_to_play[b];
    c->node_payload = s->node_payload[b];
    for (int k = 0; k < 2; ++k) {
      c->value_prior[k] = s->value_prior[2 * b + k];
      c->value_alpha[k] = s->value_alpha[2 * b + k];
    }
    for (int a = 0; a < A; ++a) {
      size_t i = (size_t)b * A + a;
      for (int k = 0; k < 2; ++k) {
        c->edge_alpha[2 * a + k] = s->edge_alpha[2 * i + k];
        c->child_prior[2 * a + k] = s->child_prior[2 * i + k];
        c->child_value[2 * a + k] = s->child_value[2 * i + k];
      }
      c->edge_payload[a] = s->edge_payload[i];
      c->edge_outcome[a] = s->edge_outcome[i];
      c->invalid[a] = s->invalid[i];
      c->child_visited[a] = s->child_visited[i];
      c->child_payload[a] = s->child_payload[i];
      c->child_outcome[a] = s->child_outcome[i];
      c->child_to_play[a] = s->child_to_play[i];
    }
    posterior_update_lane(key, c, A, u, b, B, o);
    for (int a = 0; a < A; ++a) {
      size_t i = (size_t)b * A + a;
      out_edge_alpha[2 * i] = o->edge_alpha[2 * a];
      out_edge_alpha[2 * i + 1] = o->edge_alpha[2 * a + 1];
      out_edge_payload[i] = o->edge_payload[a];
    }
    out_value_alpha[2 * b] = o->value_alpha[0];
    out_value_alpha[2 * b + 1] = o->value_alpha[1];
    out_unsafe[b] = o->unsafe;
  }
  free(c);
  free(o);
}

/* categorize + publish on explicit node indices (utils.py:67-124) */
void or_categorize_and_publish(or_tree *t, const int32_t *node, const uint8_t *active) {
  for (int b = 0; b < t->B; ++b)
    if (active[b]) categorize_and_publish(t, b, node[b]);
}

/* ------------------------------------------------------------------ */
/* synthetic game evaluation (the isolated search-kernel workload)      */
/* ------------------------------------------------------------------ */

static void synthetic_eval(const se_params *p, se_state s, int lane, float *value, float *action_values,
                           uint8_t *invalid, float *logits) {
  const int A = p->num_actions;
  int deg = se_degenerate_lane(p, lane);
  int any_legal = 0, argmin = 0;
  float umin = SM_INF;
  for (int a = 0; a < A; ++a) {
    float u = se_legal_u(s, a);
    invalid[a] = !(u < p->legal_prob);
    any_legal |= !invalid[a];
    if (u < umin) {
      umin = u;
      argmin = a;
    }
  }
  if (!any_legal) invalid[argmin] = 0;
  for (int o = 0; o < 2; ++o) value[o] = se_value_alpha(p, s, o, deg);
  for (int a = 0; a < A; ++a)
    for (int o = 0; o < 2; ++o) action_values[2 * a + o] = se_q_alpha(p, s, a, o, deg);
  if (logits)
    for (int a = 0; a < A; ++a) logits[a] = se_logit(s, a);
}

/* root network outputs + states for B lanes */
void or_synthetic_root(const se_params *p, int B, int lane_offset, float *logits, float *value,
                       float *action_values, uint8_t *invalid, int8_t *terminal, int32_t *to_play,
                       uint8_t *embedding) {
  const int A = p->num_actions;
  for (int b = 0; b < B; ++b) {
    se_state s = se_root_state(p, b + lane_offset);
    synthetic_eval(p, s, b + lane_offset, value + 2 * b, action_values + (size_t)b * A * 2,
                   invalid + (size_t)b * A, logits + (size_t)b * A);
    terminal[b] = (int8_t)se_terminal(p, s);
    to_play[b] = s.to_play;
    memcpy(embedding + (size_t)b * sizeof(se_state), &s, sizeof(se_state));
  }
}

/* recurrent_fn of the synthetic game: (parent embedding, action) -> step */
void or_synthetic_recurrent(const se_params *p, int B, int lane_offset, const int32_t *action,
                            const uint8_t *parent_embedding, float *value, float *action_values, uint8_t *invalid,
                            int8_t *terminal, int32_t *to_play, uint8_t *child_embedding) {
  const int A = p->num_actions;
  for (int b = 0; b < B; ++b) {
    se_state ps;
    memcpy(&ps, parent_embedding + (size_t)b * sizeof(se_state), sizeof(se_state));
    se_state s = se_child_state(ps, action[b]);
    synthetic_eval(p, s, b + lane_offset, value + 2 * b, action_values + (size_t)b * A * 2,
                   invalid + (size_t)b * A, NULL);
    terminal[b] = (int8_t)se_terminal(p, s);
    to_play[b] = s.to_play;
    memcpy(child_embedding + (size_t)b * sizeof(se_state), &s, sizeof(se_state));
  }
}

/* The whole dirichlet_thompson_policy (policies.py:17-48) with the search
 * loop of search.py:189-251 on the synthetic game.  The tree must be
 * allocated with emb_bytes = 16 and C = num_simulations + 1.  Returns the
 * number of prefix-CDF node updates that fell back to Monte Carlo. */
long or_search_synthetic(const se_params *p, or_tree *t, uint32_t k0, uint32_t k1, int num_simulations,
                         int max_depth, const or_update_params *u, int policy_samples,
                         const uint8_t *root_invalid, float *weights, int32_t *action) {
  const int B = t->B, A = t->A;
  sk_key rng = {k0, k1};
  sk_key search_key = sk_split(rng, 0), policy_key = sk_split(rng, 1);
  float *logits = (float *)malloc(sizeof(float) * B * A);
  float *value = (float *)malloc(sizeof(float) * B * 2);
  float *qv = (float *)malloc(sizeof(float) * B * A * 2);
  uint8_t *inv = (uint8_t *)malloc((size_t)B * A);
  int8_t *term = (int8_t *)malloc(B);
  int32_t *tp = (int32_t *)malloc(sizeof(int32_t) * B);
  uint8_t *emb = (uint8_t *)malloc((size_t)B * 16);
  uint8_t *child_emb = (uint8_t *)malloc((size_t)B * 16);
  int32_t *sp = (int32_t *)malloc(sizeof(int32_t) * B);
  int32_t *sa = (int32_t *)malloc(sizeof(int32_t) * B);
  uint8_t *sact = (uint8_t *)malloc(B);
  or_synthetic_root(p, B, t->lane_offset, logits, value, qv, inv, term, tp, emb);
  /* the root mask must outlive the loop, which reuses `inv` for each step */
  uint8_t *rinv = (uint8_t *)malloc((size_t)B * A);
  memcpy(rinv, root_invalid ? root_invalid : inv, (size_t)B * A);
  or_tree_init(t, value, qv, rinv, term, tp, emb);
  long unsafe = 0;
  sk_key key = search_key;
  for (int i = 0; i < num_simulations; ++i) {
    sk_key next = sk_split(key, 0), sim_key = sk_split(key, 1), bwd_key = sk_split(key, 3);
    or_simulate(t, sim_key, max_depth, sp, sa, sact);
    for (int b = 0; b < B; ++b) {
      int parent = sact[b] ? sp[b] : 0;
      memcpy(emb + (size_t)b * 16, t->embedding + ((size_t)b * t->C + parent) * 16, 16);
      sa[b] = sact[b] ? sa[b] : 0;
    }
    or_synthetic_recurrent(p, B, t->lane_offset, sa, emb, value, qv, inv, term, tp, child_emb);
    or_expand(t, i + 1, sp, sa, sact, value, qv, inv, term, tp, child_emb);
    unsafe += or_backward(t, bwd_key, sp, sa, sact, value, tp, u);
    key = next;
  }
  or_root_policy(t, policy_key, rinv, policy_samples, weights, action);
  free(rinv);
  free(logits);
  free(value);
  free(qv);
  free(inv);
  free(term);
  free(tp);
  free(emb);
  free(child_emb);
  free(sp);
  free(sa);
  free(sact);
  return unsafe;
}

/* ------------------------------------------------------------------ */
/* play_search.py root readout for the numerical posterior update       */
/* ------------------------------------------------------------------ */

/* _normalize_policy_on_support, play_search.py:263-295 */
static void normalize_on_support(const float *policy, const uint8_t *support, int A, float temperature,
                                 float *out) {
  float masked[MAX_ACTIONS];
  uint8_t positive[MAX_ACTIONS];
  int has_positive = 0, count = 0;
  float mx = -SM_INF;
  int mx_nan = 0;
  for (int a = 0; a < A; ++a) {
    positive[a] = support[a] && policy[a] > 0.0f;
    has_positive |= positive[a];
    count += support[a];
    float c = policy[a] > SM_TINY ? policy[a] : SM_TINY;
    if (sm_isnan(policy[a])) c = policy[a];
    c = c < 1.0f ? c : 1.0f;
    masked[a] = positive[a] ? sm_logf(c) : SM_FMIN;
    if (sm_isnan(masked[a])) mx_nan = 1;
    if (masked[a] > mx) mx = masked[a];
  }
  if (mx_nan) mx = SM_NAN;
  float scaled[MAX_ACTIONS];
  float smax = -SM_INF;
  int s_nan = 0;
  for (int a = 0; a < A; ++a) {
    scaled[a] = positive[a] ? (masked[a] - mx) / temperature : SM_FMIN;
    if (sm_isnan(scaled[a])) s_nan = 1;
    if (scaled[a] > smax) smax = scaled[a];
  }
  if (s_nan) smax = SM_NAN;
  float e[MAX_ACTIONS] = {0};
  for (int a = 0; a < A; ++a) e[a] = sm_expf(scaled[a] - smax);
  float total = warp_order_sum(e, A);
  float den = (float)(count > 1 ? count : 1);
  for (int a = 0; a < A; ++a) {
    float nrm = positive[a] ? e[a] / total : 0.0f;
    out[a] = has_positive ? nrm : (support[a] ? 1.0f : 0.0f) / den;
  }
}

/* _dirichlet_root_policy_readout with the numerical update
 * (play_search.py:161-229, 232-260, 298-364), one lane at a time. */
void or_root_readout(int B, int A, const float *native, const float *visit_counts, const float *alpha,
                     const int8_t *q_outcome, const int32_t *q_distance, const int8_t *v_outcome,
                     const uint8_t *legal, int support_search_evidence, float temperature,
                     const or_prefix_params *prm, float density_tol, float *target, uint8_t *accepted_out) {
  float pol[MAX_ACTIONS], est[MAX_ACTIONS], raw[MAX_ACTIONS], dli[MAX_ACTIONS];
  uint8_t support[MAX_ACTIONS], inv[MAX_ACTIONS], tied[MAX_ACTIONS];
  for (int b = 0; b < B; ++b) {
    const size_t r = (size_t)b * A;
    int any_candidate = 0, has_legal = 0;
    for (int a = 0; a < A; ++a) {
      int cand = legal[r + a] && (visit_counts[r + a] > 0.0f || q_outcome[r + a] != NO_OUTCOME);
      support[a] = cand;
      any_candidate |= cand;
      has_legal |= legal[r + a];
    }
    if (!support_search_evidence || !any_candidate)
      for (int a = 0; a < A; ++a) support[a] = legal[r + a];
    int has_support = 0;
    for (int a = 0; a < A; ++a) {
      inv[a] = !support[a];
      has_support |= support[a];
    }
    normalize_on_support(native + r, support, A, 1.0f, pol);
    /* _numerical_policy_readout */
    float mass, nerr, hr;
    uint8_t finite, clipped;
    int32_t fic;
    or_prefix_out po = {est, raw, &mass, &nerr, &finite, &hr, &clipped, dli, &fic};
    prefix_cdf_lane(alpha + 2 * r, inv, q_outcome + r, A, prm, &po, 0);
    float derr = 0.0f;
    int derr_nan = 0;
    for (int a = 0; a < A; ++a) {
      float v = fabsf(dli[a]);
      if (sm_isnan(v)) derr_nan = 1;
      if (v > derr) derr = v;
    }
    int unsafe = clipped || !finite || (!derr_nan && derr > density_tol);
    int root_cat = v_outcome[b] != NO_OUTCOME;
    int accepted = has_support && !root_cat && !unsafe;
    accepted_out[b] = (uint8_t)accepted;
    float tgt[MAX_ACTIONS];
    for (int a = 0; a < A; ++a) tgt[a] = accepted ? est[a] : pol[a];
    /* categorical_action_population */
    int count = categorical_candidates(v_outcome[b], q_outcome + r, q_distance + r, inv, A, tied);
    float cden = (float)(count > 1 ? count : 1);
    float cat_sum = 0.0f;
    float cat[MAX_ACTIONS];
    for (int a = 0; a < A; ++a) cat[a] = (tied[a] ? 1.0f : 0.0f) / cden;
    cat_sum = warp_order_sum(cat, A);
    if (root_cat && has_legal && cat_sum > 0.0f)
      for (int a = 0; a < A; ++a) tgt[a] = cat[a];
    normalize_on_support(tgt, support, A, temperature, target + r);
  }
}

/* ------------------------------------------------------------------ */
/* action commitment (play_search.py:627-705, dirichlet_q_search.py:79-116) */
/* ------------------------------------------------------------------ */

/* _dirichlet_commitment_policy for one batch: `sampled` is
 * posterior_best_policy over the commitment support with the commitment
 * key; a categorical root takes the one-hot of the search action; the
 * native policy is normalised on the support, and with the numerical
 * update the safe Q21 estimate replaces it (_numerical_policy_readout). */
void or_commitment_policy(int B, int A, const float *sampled, const int32_t *search_action, const float *alpha,
                          const int8_t *q_outcome, const int8_t *v_outcome, const uint8_t *legal,
                          const uint8_t *evidence, int search_evidence, int numerical, const or_prefix_params *prm,
                          float *policy) {
  float nat[MAX_ACTIONS], est[MAX_ACTIONS], raw[MAX_ACTIONS], dli[MAX_ACTIONS];
  uint8_t support[MAX_ACTIONS], inv[MAX_ACTIONS];
  for (int b = 0; b < B; ++b) {
    const size_t r = (size_t)b * A;
    const int root_cat = v_outcome[b] != NO_OUTCOME;
    int any_candidate = 0;
    for (int a = 0; a < A; ++a) {
      nat[a] = root_cat ? (a == search_action[b] ? 1.0f : 0.0f) : sampled[r + a];
      int cand = legal[r + a] && (evidence[r + a] || q_outcome[r + a] != NO_OUTCOME);
      support[a] = cand;
      any_candidate |= cand;
    }
    if (!search_evidence || !any_candidate)
      for (int a = 0; a < A; ++a) support[a] = legal[r + a];
    int has_support = 0;
    for (int a = 0; a < A; ++a) {
      inv[a] = !support[a];
      has_support |= support[a];
    }
    normalize_on_support(nat, support, A, 1.0f, policy + r);
    if (!numerical) continue;
    float mass, nerr, hr;
    uint8_t finite, clipped;
    int32_t fic;
    or_prefix_out po = {est, raw, &mass, &nerr, &finite, &hr, &clipped, dli, &fic};
    prefix_cdf_lane(alpha + 2 * r, inv, q_outcome + r, A, prm, &po, 0);
    float derr = 0.0f;
    int derr_nan = 0;
    for (int a = 0; a < A; ++a) {
      float v = fabsf(dli[a]);
      if (sm_isnan(v)) derr_nan = 1;
      if (v > derr) derr = v;
    }
    int unsafe = clipped || !finite || (!derr_nan && derr > 0.01f);
    if (has_support && !root_cat && !unsafe)
      for (int a = 0; a < A; ++a) policy[r + a] = est[a];
  }
}

/* posterior_best_action (kind 0) / posterior_sample_action (kind 1):
 * argmax of the masked policy, or jax.random.categorical(key, logits) =
 * argmax(logits + gumbel) of logits = log(clip(p, 1e-8, 1)) / T on the
 * legal actions with positive policy (all legal ones if none has); the
 * Gumbel noise is -log(-log(uniform(key, [B, A], tiny, 1))). */
void or_commit_action(int kind, uint32_t k0, uint32_t k1, const float *policy, const uint8_t *legal, int B, int A,
                      float temperature, int32_t *action) {
  float score[MAX_ACTIONS];
  sk_key key = {k0, k1};
  for (int b = 0; b < B; ++b) {
    const size_t r = (size_t)b * A;
    int any_pos = 0;
    for (int a = 0; a < A; ++a) any_pos |= legal[r + a] && policy[r + a] > 0.0f;
    for (int a = 0; a < A; ++a) {
      const float p = policy[r + a];
      if (kind == 0) {
        score[a] = legal[r + a] ? p : -SM_INF;
        continue;
      }
      const int eligible = any_pos ? (legal[r + a] && p > 0.0f) : legal[r + a];
      float c = p > 1e-8f ? p : 1e-8f;
      if (sm_isnan(p)) c = p;
      c = c < 1.0f ? c : 1.0f;
      const float logit = eligible ? sm_logf(c) / temperature : SM_FMIN;
      const float u = sk_uniform(key, (uint64_t)b * A + a, SM_TINY, 1.0f);
      score[a] = logit + (-sm_logf(-sm_logf(u)));
    }
    action[b] = nan_first_argmax(score, A);
  }
}
