/*
 * Seeded synthetic game for the isolated search-kernel workload: Hex 9x9
 * action space (82 actions), network outputs synthesised from the seed.
 *
 * A state is a threefry key plus the player to move; taking action `a`
 * folds `a` into the key and flips the player, so every path through the
 * tree names a distinct, reproducible state.  The "network" reads the key:
 *   prior logits            N(0, 1)                      fold_in(state, 2)
 *   value log-concentration clip(mean + std N(0,1), lo, hi) per outcome,
 *                           alpha = exp(.)               fold_in(state, 3)
 *   Q log-concentrations    same, per (action, outcome)  fold_in(state, 4)
 *   legal mask              U(0,1) < legal_prob, and the first minimum of U
 *                           is legal when no draw passes fold_in(state, 1)
 *   terminal (depth >= 1)   U(0,1) < terminal_prob, outcome = one random bit
 *                                                        fold_in(state, 5)
 * A lane is near-degenerate with probability degenerate_lane_prob
 * (U(0,1) at index `lane` of fold_in(seed, 1)); all of its concentrations
 * are then `degenerate_alpha`.
 *
 * Shared by the CUDA synthetic evaluator and the C oracle: it generates the
 * test input, it is not part of the algorithm under test.
 */
#ifndef SCACCHI_SYNTHETIC_ENV_H
#define SCACCHI_SYNTHETIC_ENV_H

#include "threefry.h"

typedef struct {
  uint32_t seed_k0, seed_k1;
  int32_t num_actions;
  float legal_prob;
  float terminal_prob;
  float degenerate_lane_prob;
  float degenerate_alpha;
  float logc_mean, logc_std, logc_min, logc_max;
} se_params;

/* 16-byte per-node embedding stored in the tree */
typedef struct {
  uint32_t k0, k1;
  int32_t to_play;
  int32_t depth;
} se_state;

SM_FN sk_key se_seed(const se_params *p) {
  sk_key k;
  k.k0 = p->seed_k0;
  k.k1 = p->seed_k1;
  return k;
}

SM_FN se_state se_root_state(const se_params *p, int lane) {
  sk_key k = sk_fold_in(sk_fold_in(se_seed(p), 2u), (uint32_t)lane);
  se_state s;
  s.k0 = k.k0;
  s.k1 = k.k1;
  s.to_play = 0;
  s.depth = 0;
  return s;
}

SM_FN se_state se_child_state(se_state parent, int action) {
  sk_key k;
  k.k0 = parent.k0;
  k.k1 = parent.k1;
  sk_key c = sk_fold_in(k, (uint32_t)action);
  se_state s;
  s.k0 = c.k0;
  s.k1 = c.k1;
  s.to_play = 1 - parent.to_play;
  s.depth = parent.depth + 1;
  return s;
}

SM_FN sk_key se_stream(se_state s, uint32_t which) {
  sk_key k;
  k.k0 = s.k0;
  k.k1 = s.k1;
  return sk_fold_in(k, which);
}

SM_FN int se_degenerate_lane(const se_params *p, int lane) {
  return sk_uniform(sk_fold_in(se_seed(p), 1u), (uint64_t)lane, 0.0f, 1.0f) < p->degenerate_lane_prob;
}

SM_FN float se_legal_u(se_state s, int a) {
  return sk_uniform(se_stream(s, 1u), (uint64_t)a, 0.0f, 1.0f);
}

SM_FN float se_logit(se_state s, int a) { return sk_normal(se_stream(s, 2u), (uint64_t)a); }

SM_FN float se_concentration(const se_params *p, sk_key stream, uint64_t i, int degenerate) {
  if (degenerate) return p->degenerate_alpha;
  float c = p->logc_mean + p->logc_std * sk_normal(stream, i);
  c = c > p->logc_min ? c : p->logc_min;
  c = c < p->logc_max ? c : p->logc_max;
  return sm_expf(c);
}

SM_FN float se_value_alpha(const se_params *p, se_state s, int o, int degenerate) {
  return se_concentration(p, se_stream(s, 3u), (uint64_t)o, degenerate);
}

SM_FN float se_q_alpha(const se_params *p, se_state s, int a, int o, int degenerate) {
  return se_concentration(p, se_stream(s, 4u), (uint64_t)a * 2u + (uint64_t)o, degenerate);
}

/* exact terminal outcome from the state's own to_play perspective, or -1 */
SM_FN int se_terminal(const se_params *p, se_state s) {
  if (s.depth == 0) return -1;
  sk_key k = se_stream(s, 5u);
  if (!(sk_uniform(k, 0u, 0.0f, 1.0f) < p->terminal_prob)) return -1;
  return (int)(sk_bits(k, 1u) & 1u);
}

#endif /* SCACCHI_SYNTHETIC_ENV_H */
