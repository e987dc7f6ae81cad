/*
 * scacchi_b200 — C ABI of the B200 Dirichlet-Thompson search step.
 *
 * Every entry point takes device pointers, plain sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns an
 * int status: 0 = ok, SCACCHI_EINVAL = rejected arguments (nothing was
 * launched), SCACCHI_ECUDA = a CUDA launch error.  Device-side index checks
 * (a tree index outside [0, num_nodes)) skip the access and raise a sticky
 * flag read by scacchi_device_error().
 *
 * The reference (Francesco215/Scacchi) is pure Python/JAX; each entry point
 * below names the function of `scacchi/dirichlet_mctx` (or of
 * `scacchi/play_search.py`) whose semantics it implements and that a jax.ffi
 * custom call would bind to.  Outcomes are binary (loss 0, win 1): the Hex
 * configuration.  Actions per node: 1 <= num_actions <= 128.
 *
 * Tree layout (struct of arrays, lanes outermost, C = num_nodes,
 * S = action_stride = num_actions rounded up to a multiple of 32):
 *   parents, node_to_play, node_payload   int32   [B, C]
 *   node_outcome                          int8    [B, C]
 *   node_value_prior, node_value_alpha    float32 [B, C, 2]
 *   children_index, edge_payload          int32   [B, C, S]
 *   edge_outcome                          int8    [B, C, S]
 *   invalid                               uint8   [B, C, S]
 *   edge_alpha                            float32 [B, C, S, 2]
 *   embedding                             uint8   [B, C, emb_bytes]
 * Per-lane inputs and outputs use dense [B, A] rows.
 *
 * Keys are jax.random threefry key pairs (uint32[2]) in device memory.
 */
#ifndef SCACCHI_B200_H
#define SCACCHI_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SCACCHI_OK 0
#define SCACCHI_EINVAL 1
#define SCACCHI_ECUDA 2
#define SCACCHI_ETOOLARGE 3 /* larger than a fixed library-owned buffer */

typedef struct {
  int32_t batch;
  int32_t num_nodes;
  int32_t num_actions;
  int32_t action_stride;
  int32_t emb_bytes;
  int32_t *parents;
  int32_t *children_index;
  int32_t *node_to_play;
  int8_t *node_outcome;
  int32_t *node_payload;
  int8_t *edge_outcome;
  int32_t *edge_payload;
  float *node_value_prior;
  float *node_value_alpha;
  float *edge_alpha;
  uint8_t *invalid;
  uint8_t *embedding;
} scacchi_tree;

/* Static parameters of the two built-in posterior repair rules
 * (posterior_updates.py:220-367). */
typedef struct {
  int32_t rule;              /* 0: update_posterior (Monte Carlo), 1: update_posterior_prefix_cdf */
  int32_t kappa_ge_one;      /* kappa >= 1, decided in double precision */
  float inv_kappa;           /* float32(1 / kappa) */
  float kappa;               /* float32(kappa), read only when kappa < 1 */
  int32_t samples;           /* policy_samples (rule 0) / fallback_policy_samples (rule 1) */
  int32_t half_width;        /* Q = 2 * half_width + 1 grid points */
  float tail_scale;
  float min_half_range;
  float max_half_range;
  float density_tol;         /* density_log_integral_tolerance */
} scacchi_update_params;

/* Prefix-CDF estimator outputs (BinaryPrefixQuadraturePolicy, prefix_cdf.py:21-37). */
typedef struct {
  float *policy;                   /* [B, A] */
  float *raw_policy;               /* [B, A] */
  float *raw_mass;                 /* [B] */
  float *normalization_error;      /* [B] */
  uint8_t *finite;                 /* [B] */
  float *grid_half_range;          /* [B] */
  uint8_t *tail_range_clipped;     /* [B] */
  float *density_log_integral;     /* [B, A] */
  int32_t *fallback_interval_count;/* [B] */
} scacchi_prefix_out;

/* Synthetic-game parameters (isolated search-kernel workload). */
typedef struct {
  uint32_t seed_k0, seed_k1;
  int32_t num_actions;
  float legal_prob;
  float terminal_prob;
  float degenerate_lane_prob;
  float degenerate_alpha;
  float logc_mean, logc_std, logc_min, logc_max;
} scacchi_synthetic_params;

/* ---- search core (scacchi/dirichlet_mctx) ---------------------------- */

/* instantiate_tree_from_root (tree.py:245-277).  full_init != 0 writes the
 * defaults of every node slot; full_init == 0 writes only the root row and
 * leaves slots 1..C-1 to scacchi_expand(lazy_init=1), which writes each slot
 * exactly once, before any read.  root_embedding may be NULL. */
int scacchi_tree_init(const scacchi_tree *tree, const float *root_value, const float *root_action_values,
                      const uint8_t *root_invalid, const int8_t *root_terminal, const int32_t *root_to_play,
                      const uint8_t *root_embedding, int32_t full_init, void *stream);

/* simulate / _simulate_one (search.py:21-78): one warp per lane walks the
 * tree with Thompson selection until an unvisited edge, a categorical or
 * unsearchable child, or max_depth.  simulate_key: uint32[2].  When
 * parent_embedding is non-NULL the selected parent's embedding row is
 * gathered into it ([B, emb_bytes]).  stats (may be NULL) accumulates
 * uint64[2]: nodes selected from, child value priors gathered. */
int scacchi_simulate(const scacchi_tree *tree, const uint32_t *simulate_key, int32_t max_depth,
                     int32_t *parent, int32_t *action, uint8_t *active, uint8_t *parent_embedding,
                     uint64_t *stats, void *stream);

/* expand (search.py:101-143).  step_* are the recurrent_fn outputs
 * (RecurrentFnOutput, base.py:58-74); child_embedding may be NULL.
 * lazy_init != 0 also writes the defaults of slot new_node for lanes that do
 * not initialise it (see scacchi_tree_init). */
int scacchi_expand(const scacchi_tree *tree, int32_t new_node, const int32_t *parent, const int32_t *action,
                   const uint8_t *active, const float *step_value, const float *step_action_values,
                   const uint8_t *step_invalid, const int8_t *step_terminal, const int32_t *step_to_play,
                   const uint8_t *child_embedding, int32_t lazy_init, void *stream);

/* backward (search.py:146-171) with the posterior update rule of `params`
 * (update_posterior / update_posterior_prefix_cdf, posterior_updates.py)
 * and _categorize_node_and_publish (utils.py:67-124).  stats (may be NULL)
 * accumulates uint64[3]: node updates, visited children gathered,
 * prefix-CDF updates that fell back to Monte Carlo. */
int scacchi_backward(const scacchi_tree *tree, const uint32_t *backward_key, const int32_t *parent,
                     const int32_t *action, const uint8_t *active, const float *step_value,
                     const int32_t *step_to_play, const scacchi_update_params *params,
                     uint64_t *stats, void *stream);

/* dirichlet_thompson_policy root readout (policies.py:28-42): one-hot on the
 * sampled certified action of a categorical root, else posterior_best_policy
 * with max(1, policy_samples) draws; then masked_argmax. */
int scacchi_root_policy(const scacchi_tree *tree, const uint32_t *policy_key, const uint8_t *invalid,
                        int32_t policy_samples, float *action_weights, int32_t *action, void *stream);

/* Tree.summary (tree.py:212-242). */
int scacchi_summary(const scacchi_tree *tree, float *visit_counts, float *alpha, float *value_alpha,
                    int8_t *q_outcome, int32_t *q_distance, int8_t *v_outcome, int32_t *v_distance,
                    void *stream);

/* ---- estimators ------------------------------------------------------- */

/* binary_posterior_best_policy_prefix_quadrature (prefix_cdf.py:217-445)
 * on alpha [B, A, 2]; categorical_outcome may be NULL (all unresolved). */
int scacchi_prefix_cdf(const float *alpha, const uint8_t *invalid, const int8_t *categorical_outcome,
                       int32_t batch, int32_t num_actions, int32_t half_width, float tail_scale,
                       float min_half_range, float max_half_range, const scacchi_prefix_out *out,
                       void *stream);

/* posterior_best_policy (action_selection.py:146-194) on alpha [B, A, 2];
 * categorical_outcome may be NULL. */
int scacchi_posterior_best_policy(const uint32_t *key, const float *alpha, const uint8_t *invalid,
                                  const int8_t *categorical_outcome, int32_t batch, int32_t num_actions,
                                  int32_t num_samples, float *policy, void *stream);

/* thompson_sample (action_selection.py:135-143) on alpha [B, A, 2]. */
int scacchi_thompson_sample(const uint32_t *key, const float *alpha, const uint8_t *invalid,
                            const int8_t *categorical_outcome, int32_t batch, int32_t num_actions,
                            int32_t *action, void *stream);

/* update_posterior / update_posterior_prefix_cdf on explicit contexts
 * (PosteriorUpdateContext, tree.py:30-83), struct-of-arrays with a leading
 * batch axis; the field order is that of scacchi_context below. */
typedef struct {
  const uint8_t *active;
  const uint8_t *leaf_active;
  const int32_t *leaf_action;
  const float *leaf_value;
  const int32_t *leaf_to_play;
  const int32_t *node_to_play;
  const int32_t *node_payload;
  const float *value_prior;
  const float *value_alpha;
  const float *edge_alpha;
  const int32_t *edge_payload;
  const int8_t *edge_outcome;
  const uint8_t *invalid;
  const uint8_t *child_visited;
  const float *child_prior;
  const float *child_value;
  const int32_t *child_payload;
  const int8_t *child_outcome;
  const int32_t *child_to_play;
} scacchi_context;

int scacchi_update_posterior(const uint32_t *key, const scacchi_context *context, int32_t batch,
                             int32_t num_actions, const scacchi_update_params *params, float *edge_alpha,
                             int32_t *edge_payload, float *value_alpha, uint8_t *unsafe, void *stream);

/* ---- search boundary (scacchi/play_search.py) ------------------------- */

/* _dirichlet_root_policy_readout with the numerical update
 * (play_search.py:161-364): search-evidence support, Q21 readout with the
 * native fallback, categorical population, power-temperature
 * renormalisation.  All inputs are the root summary ([B, A] / [B]). */
int scacchi_root_readout(int32_t batch, int32_t num_actions, const float *native_policy,
                         const float *visit_counts, const float *alpha, const int8_t *q_outcome,
                         const int32_t *q_distance, const int8_t *v_outcome, const uint8_t *legal,
                         int32_t search_evidence_support, float temperature, int32_t half_width,
                         float tail_scale, float min_half_range, float max_half_range, float *policy_target,
                         uint8_t *accepted, void *stream);

/* _dirichlet_commitment_policy (play_search.py:627-705): the root policy
 * an action is committed from.  sampled_policy is posterior_best_policy
 * (scacchi_posterior_best_policy) over the commitment support with the
 * commitment key; a root with v_outcome != -1 takes the one-hot of
 * search_action instead.  The support is _root_policy_support of the
 * legal actions, positive_evidence ([B, A], actions with search visits)
 * and q_outcome; numerical != 0 replaces the normalised native policy by
 * the safe Q21 estimate (_numerical_policy_readout). */
int scacchi_commitment_policy(int32_t batch, int32_t num_actions, const float *sampled_policy,
                              const int32_t *search_action, const float *alpha, const int8_t *q_outcome,
                              const int8_t *v_outcome, const uint8_t *legal, const uint8_t *positive_evidence,
                              int32_t search_evidence_support, int32_t numerical, int32_t half_width,
                              float tail_scale, float min_half_range, float max_half_range, float *policy,
                              void *stream);

/* posterior_best_action (kind 0) and posterior_sample_action (kind 1,
 * power-temperature jax.random.categorical with key uint32[2]),
 * dirichlet_q_search.py:79-116. */
int scacchi_commit_action(int32_t kind, const uint32_t *key, const float *policy, const uint8_t *legal,
                          int32_t batch, int32_t num_actions, float temperature, int32_t *action, void *stream);

/* ---- synthetic game (isolated search-kernel workload) ----------------- */

int scacchi_synthetic_root(const scacchi_synthetic_params *params, int32_t batch, float *prior_logits,
                           float *value, float *action_values, uint8_t *invalid, int8_t *terminal,
                           int32_t *to_play, uint8_t *embedding, void *stream);

/* Network outputs of given states ([B, 16] bytes), no step. */
int scacchi_synthetic_evaluate(const scacchi_synthetic_params *params, int32_t batch, const uint8_t *states,
                               float *prior_logits, float *value, float *action_values, uint8_t *invalid,
                               int8_t *terminal, int32_t *to_play, void *stream);

int scacchi_synthetic_recurrent(const scacchi_synthetic_params *params, int32_t batch, const int32_t *action,
                                const uint8_t *parent_embedding, float *value, float *action_values,
                                uint8_t *invalid, int8_t *terminal, int32_t *to_play, uint8_t *child_embedding,
                                void *stream);

/* The whole simulation loop on the synthetic game (search.py:189-251):
 * for i < num_simulations: simulate, recurrent, expand(lazy), backward.
 * `keys` holds the per-simulation key schedule uint32[num_simulations, 4, 2]
 * (split(key, 4) chain), `workspace` at least scacchi_search_workspace_bytes()
 * bytes of device memory.  The tree root must already be initialised. */
size_t scacchi_search_workspace_bytes(int32_t batch, int32_t num_actions, int32_t emb_bytes);
/* stats (may be NULL): uint64[6] = backward stats [0..2], unused [3],
 * simulate stats [4..5]. */
int scacchi_search_synthetic(const scacchi_tree *tree, const scacchi_synthetic_params *env,
                             const uint32_t *keys, int32_t num_simulations, int32_t max_depth,
                             const scacchi_update_params *params, void *workspace, uint64_t *stats,
                             void *stream);

/* No counterpart in the reference.  scacchi_search_synthetic for callers
 * that cannot allocate device memory at call time (an XLA FFI handler,
 * whose allocator owns the device's memory and offers scratch only as
 * declared buffers; a server that pins all of HBM to a pool at start-up).
 * Instead of a caller workspace it uses a scratch array compiled into the
 * library: SCACCHI_STATIC_SCRATCH_BYTES per device, held by every GPU that
 * loads the library until the process exits.  The caller still passes the
 * tree, keys and stats.  It calls no cudaMalloc, cudaFree or allocating
 * library routine.
 *   - Sizes whose workspace (scacchi_search_workspace_bytes) exceeds the
 *     array return SCACCHI_ETOOLARGE; nothing is launched.  At 82 actions
 *     and 16-byte states the limit is 5,294 lanes.
 *   - The first call on a device resolves the array's device address with
 *     that device current (cudaGetSymbolAddress); make that first call
 *     before any stream capture on the device.  The address is kept with
 *     the context it was resolved in: after the context is torn down and
 *     created again (cudaDeviceReset) the next call resolves it again, so
 *     that call too belongs before any capture.
 *   - A malformed descriptor returns SCACCHI_EINVAL before the size is
 *     looked at.
 *   - All calls on a device share the one array, which keeps the last
 *     call's contents.  Calls whose work overlaps on the GPU (different
 *     streams, or different host threads without ordering) race on it and
 *     corrupt each other's results: order them on one stream. */
#define SCACCHI_STATIC_SCRATCH_BYTES (4u << 20)
int scacchi_search_synthetic_static(const scacchi_tree *tree, const scacchi_synthetic_params *env,
                                    const uint32_t *keys, int32_t num_simulations, int32_t max_depth,
                                    const scacchi_update_params *params, uint64_t *stats, void *stream);

/* ---- Hex environment (envs.py:98-125 over pgx 2.6.0 Hex) -------------- */

/* A lane's state is a 48-byte record: black and white bitboards (bit
 * r * size + c of two little-endian uint64 words each), then colour to move
 * (0 black), the player id playing black, terminated, the winning colour
 * (int8, -1 none), size and stones placed.  Actions are the size * size
 * cells plus a swap action (index size * size) that is never legal.
 * Observations are float32 [B, size, size, 4] for the player to move: own
 * stones, opponent stones, own colour, 1 on the second move. */
#define SCACCHI_HEX_RECORD_BYTES 48

/* env.init (envs.py:103-112) per lane key uint32[B, 2]. */
int scacchi_hex_init(int32_t batch, int32_t size, const uint32_t *keys, uint8_t *states, void *stream);

/* Seeded roots of the full-step workload: per lane, a random player order
 * and min_moves..max_moves uniform random legal moves from the empty
 * board (no reference counterpart). */
int scacchi_hex_random_roots(int32_t batch, int32_t size, uint32_t key0, uint32_t key1, int32_t min_moves,
                             int32_t max_moves, uint8_t *states, void *stream);

/* env.step (envs.py:114-123) fused with the recurrent function's
 * derivations (dirichlet_q_search.py:43-76): next_states [B, 48] and,
 * for each non-NULL output, the child's observation, invalid actions
 * [B, size*size + 1], terminal outcome aligned to the child's player (-1
 * when not terminal), player to move, rewards [B, 2] and terminated.  An
 * illegal action or a terminal parent leaves the state unchanged (the
 * search steps lanes with nothing to expand with action 0 and discards
 * their results); a record whose size is out of range sets bit 0 of
 * scacchi_hex_error() and writes nothing for that lane. */
int scacchi_hex_step(int32_t batch, const uint8_t *states, const int32_t *action, uint8_t *next_states,
                     float *observation, uint8_t *invalid, int8_t *terminal_outcome, int32_t *to_play,
                     float *rewards, uint8_t *terminated, void *stream);

/* The same outputs for given states (roots): the terminal outcome is from
 * the perspective of the state's own player to move. */
int scacchi_hex_observe(int32_t batch, const uint8_t *states, float *observation, uint8_t *invalid,
                        int8_t *terminal_outcome, int32_t *to_play, float *rewards, uint8_t *terminated,
                        void *stream);

/* Sticky Hex error flags (bit 0: a record with an out-of-range size;
 * reading synchronises and clears) and launches. */
int scacchi_hex_error(uint32_t *flags);
uint64_t scacchi_hex_launch_count(void);

/* ---- leaf evaluation: AZDirichletNet (network.py:338-524) -------------- */

/* Inference weights of the 9x9 resnet_v2 AZDirichletNet with binary
 * outcomes, BatchNorm in inference form (running statistics):
 *   stem_w      float32 [9 taps (ky*3+kx)][in_planes][128], stem_b [128]
 *   bn_scale/shift float32 [num_blocks + 1][128]: BN1 of every block, then
 *               the trunk's final BN, as y = x * scale + shift
 *   conv_w      16-bit [2 * num_blocks][parts][9 taps][128 out][128 in]
 *               (bf16, or fp16 when fp16 = 1), parts = 2 when terms = 3
 *               (the weight rounded to 16 bits, then the remainder rounded
 *               to 16 bits), else 1; the BN after each block's first conv
 *               is folded into that conv's weights and bias; conv_b float32
 *               [2 * num_blocks][128]
 *   head_w      float32 [6][128], head_b [6]: 1x1 convs of the policy (2),
 *               value (1), Q-mean (2) and Q-concentration (1) heads with
 *               their BNs folded
 *   dense layers as [in][out] row-major with flax's flatten order
 *               (y, x, channel). */
typedef struct {
  int32_t num_blocks, channels, height, width, in_planes, num_actions;
  int32_t fp16;  /* 16-bit operand and activation type: 0 bf16, 1 fp16 */
  /* tensor-core products per K step: 1 = 16-bit activations and weights,
   * 16-bit residual stream (the reference's bf16 model); 2 = activations
   * split into hi + lo 16-bit matrices (A_hi W + A_lo W); 3 = weights split
   * too (+ A_hi W_lo).  With 2 or 3 the residual stream stays fp32. */
  int32_t terms;
  const float *stem_w, *stem_b;
  const float *bn_scale, *bn_shift;
  const uint16_t *conv_w;
  const float *conv_b;
  const float *head_w, *head_b;
  const float *policy_w, *policy_b;          /* [162][A], [A] */
  const float *value_w1, *value_b1;          /* [81][128], [128] */
  const float *value_mean_w, *value_mean_b;  /* [128][2], [2] */
  const float *value_conc_w, *value_conc_b;  /* [128], [1] */
  const float *qdir_w1, *qdir_b1;            /* [162][128], [128] */
  const float *qdir_w2, *qdir_b2;            /* [128][2A], [2A] */
  const float *qconc_w1, *qconc_b1;          /* [81][128], [128] */
  const float *qconc_w2, *qconc_b2;          /* [128][A], [A] */
} scacchi_tower_weights;

/* Rows of one padded activation matrix for `boards` boards (100 rows per
 * board, rounded up to the 128-row tile) and the workspace the forward
 * pass needs with any `terms` (split operands: an fp32 [rows, 128] residual
 * stream and four 16-bit [rows, 128] matrices; head features). */
uint64_t scacchi_tower_rows(int32_t boards);
size_t scacchi_tower_workspace_bytes(int32_t boards);

/* AZDirichletNet.__call__(obs, train=False) (network.py:460-524): obs
 * float32 [B, 9, 9, planes] -> logits [B, A], log alpha_v [B, 2], log
 * alpha_q [B, A, 2] (log concentration + log softmax of the mean logits)
 * and the alphas themselves.  16-bit tensor-core convolutions (1, 2 or 3
 * products per K step, weights->terms), fp32 accumulation. */
int scacchi_tower_forward(const scacchi_tower_weights *weights, const float *obs, int32_t boards, void *workspace,
                          float *logits, float *log_alpha_v, float *log_alpha_q, float *alpha_v, float *alpha_q,
                          void *stream);

/* One padded-layout conv3x3 128->128 (tcgen05 implicit GEMM on 16-bit
 * operands, bf16 or fp16, fp32 accumulation) with its
 * fused epilogue: mode 0 out0 = relu(conv + bias); mode 1 out0 = x' =
 * conv + bias + residual, out1 = relu(x' * bn_scale + bn_shift); mode 2 as
 * mode 1 then the six 1x1 head channels relu(out1 . head_w + head_b) into
 * head_out float32 [rows, 8].  Padding rows are written as zero. */
int scacchi_conv3x3(const void *input, const void *weights, const float *bias, int32_t mode, int32_t boards,
                    int32_t fp16, const float *bn_scale, const float *bn_shift, const void *residual,
                    const float *head_w, const float *head_b, void *out0, void *out1, float *head_out,
                    void *stream);

/* The same convolution on split operands (terms 2 or 3): the input is the
 * pair input (hi) + input_lo of 16-bit matrices, weights [terms == 3 ? 2 :
 * 1][9][128 out][128 in], and the residual stream x32 float32 [rows, 128],
 * each row's channels permuted within their 32-channel block: channel
 * 32 q + 8 m + l (l < 8, m < 4) is stored at 32 q + 4 l + m (so an epilogue
 * thread's four channels of a row are one 16-byte vector).  With
 * x32_natural_in = 1 the input x32 is read in the natural channel order
 * (the stem's output, for the first block) and written back permuted.
 * mode 0: (out_hi, out_lo) = split(relu(conv + bias)); mode 1: x32 <- x' =
 * conv + bias + x32 (in place), (out_hi, out_lo) = split(relu(x' *
 * bn_scale + bn_shift)); mode 2: as mode 1 without the stores, then the six
 * 1x1 head channels from the fp32 activation into head_out.  split(v): hi =
 * v rounded to 16 bits, lo = (v - hi) rounded to 16 bits. */
int scacchi_conv3x3_split(const void *input, const void *input_lo, const void *weights, const float *bias,
                          int32_t mode, int32_t boards, int32_t fp16, int32_t terms, const float *bn_scale,
                          const float *bn_shift, float *x32, int32_t x32_natural_in, const float *head_w,
                          const float *head_b, void *out_hi, void *out_lo, float *head_out, void *stream);

/* Sticky tower error flags (bit 0: a bounded wait timed out); reading
 * synchronises and clears.  Launch counter of the tower kernels. */
int scacchi_tower_error(uint32_t *flags);
uint64_t scacchi_tower_launch_count(void);

/* Optional timing of the tower's convolutions (no reference counterpart:
 * measurement only).  scacchi_tower_timing(n) makes the next n forwards
 * record a CUDA event pair around their conv launches on their stream (0
 * turns it off); scacchi_tower_timing_read waits for those events and
 * returns the summed conv time (ms) and the number of forwards timed, then
 * starts counting again. */
int scacchi_tower_timing(int32_t max_forwards);
int scacchi_tower_timing_read(float *conv_ms, int32_t *forwards);

/* ---- the callers either side of the root: targets and loss input ------- */

/* _run_dirichlet_thompson_search's target packing (play_search.py:490-548)
 * with build_q_supervision (dirichlet_q_search.py:119-182), from the tree
 * summary: per [batch, num_actions] q_kind (int8: 0 pad, 1 Dirichlet, 2
 * categorical), selected, pair_weight, positive_evidence, positive_policy,
 * q_weight; per lane v_kind, v_weight and the search loss mask (sum of the
 * policy target > 0).  action_set 0 = positive search evidence or solved, 1
 * = positive posterior policy or solved; reduction 0 = mean over selected
 * pairs, 1 = legacy source-weighted.  Booleans are one byte. */
int scacchi_pack_targets(int32_t batch, int32_t num_actions, const float *visit_counts, const float *policy_target,
                         const uint8_t *legal, const int8_t *q_outcome, const int8_t *v_outcome, int32_t action_set,
                         int32_t reduction, int8_t *q_kind, int8_t *v_kind, uint8_t *mask, uint8_t *selected,
                         float *pair_weight, uint8_t *positive_evidence, uint8_t *positive_policy, float *q_weight,
                         float *v_weight, void *stream);

/* Self-play frames of `batch` trajectories x `frames_per_lane` steps, lane
 * major ([B, T] and [B, T, A]), as compute_loss_input reads them
 * (loss.py:164-357).  search_mask may be NULL (then sum of the policy > 0). */
typedef struct {
  const float *reward, *discount;      /* [B, T] */
  const uint8_t *terminated;           /* [B, T] */
  const int32_t *played_action;        /* [B, T] */
  const uint8_t *legal;                /* [B, T, A] */
  const float *policy;                 /* [B, T, A] posterior policy target */
  const uint8_t *search_mask;          /* [B, T] metadata mask, or NULL */
  const uint8_t *q_pair_mask;          /* [B, T, A] q_supervision.selected */
  const float *q_pair_weight;          /* [B, T, A] */
  const int8_t *q_kind, *q_outcome;    /* [B, T, A] native Q sidecars */
  const float *q_weight;
  const int32_t *q_distance;
  const int8_t *v_kind, *v_outcome;    /* [B, T] native V sidecars */
  const float *v_weight;
  const int32_t *v_distance;
} scacchi_loss_frames;

typedef struct {
  float *value_tgt;                    /* [B, T] trajectory value targets */
  uint8_t *value_mask, *policy_loss_mask, *value_loss_mask, *search_loss_mask;  /* [B, T] */
  float *policy_tgt;                   /* [B, T, A] */
  uint8_t *q_pair_mask;                /* [B, T, A] */
  float *q_pair_weight;
  int8_t *q_kind, *q_outcome;
  float *q_weight;
  int32_t *q_distance;
  int8_t *v_kind, *v_outcome;          /* [B, T] */
  float *v_weight;
  int32_t *v_distance;
} scacchi_loss_out;

/* The frame-wise part of compute_loss_input: the reverse value scan
 * (loss.py:231-245), the value / policy / value-loss / search-loss masks
 * of loss_mask_mode (0 search, 1 value, 2 pgx), the winner-action policy
 * target, and the exact one-step terminal targets (loss.py:117-136) on the
 * played edge (terminal_edge_targets) and on a won terminal parent
 * (terminal_parent_targets); legacy_reduction selects the legacy
 * source-weighted Q pair weight.  One CTA per trajectory. */
int scacchi_loss_input(const scacchi_loss_frames *frames, const scacchi_loss_out *out, int32_t batch,
                       int32_t frames_per_lane, int32_t num_actions, int32_t num_outcomes, int32_t loss_mask_mode,
                       int32_t winner_action_policy, int32_t terminal_edge_targets, int32_t terminal_parent_targets,
                       int32_t legacy_reduction, void *stream);
uint64_t scacchi_target_launch_count(void);

/* ---- host-side jax.random key helpers (no device work) ---------------- */

/* search.py:207-209 key chain: for i < num_simulations,
 * (key_{i+1}, simulate, expand, backward) = split(key_i, 4); key_0 is the
 * search key.  out: uint32[num_simulations, 4, 2]. */
int scacchi_key_schedule(uint32_t k0, uint32_t k1, int32_t num_simulations, uint32_t *out);
/* jax.random.split(key, n) -> out uint32[n, 2] */
int scacchi_split_host(uint32_t k0, uint32_t k1, int32_t n, uint32_t *out);
/* jax.random.fold_in(key, data) -> out uint32[2] */
int scacchi_fold_in_host(uint32_t k0, uint32_t k1, uint32_t data, uint32_t *out);

/* ---- diagnostics ------------------------------------------------------- */

/* Sticky device-side error flags (bit 0: tree index out of range); reading
 * synchronises the device and clears the flags. */
int scacchi_device_error(uint32_t *flags);

/* Number of kernels this library has launched since load (all streams). */
uint64_t scacchi_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* SCACCHI_B200_H */
