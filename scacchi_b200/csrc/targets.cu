// The callers either side of the search's root: the packing of the search's
// targets (play_search.py:490-548 with dirichlet_q_search.py:119-182) and
// the loss-input assembly of self-play frames (loss.py:117-161, 164-357,
// 412-423, 511-517).  Both are elementwise over lanes x actions plus one
// reduction over actions (the targets) or one reverse scan over time (the
// frames); each runs as one launch.
//
// Compiled with -fmad=false: value targets are r + d * v with the product
// and the sum rounded separately, as the reference's jnp expression.

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/scacchi_b200.h"

namespace {

constexpr int kTargetPad = 0, kTargetDirichlet = 1, kTargetCategorical = 2;
constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

std::atomic<uint64_t> g_target_launches{0};

// One warp per lane: the actions in chunks of 32.  q_kind / q_weight /
// selected / pair_weight / positive masks per action; v_kind, v_weight and
// the search loss mask (sum over actions of the policy target > 0) per lane.
__global__ void pack_targets_kernel(int B, int A, const float *visit, const float *policy, const uint8_t *legal,
                                    const int8_t *q_outcome, const int8_t *v_outcome, int action_set, int reduction,
                                    int8_t *q_kind, int8_t *v_kind, uint8_t *mask, uint8_t *selected,
                                    float *pair_weight, uint8_t *pos_evidence, uint8_t *pos_policy, float *q_weight,
                                    float *v_weight) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarp, lane = threadIdx.x % kWarp;
  if (warp >= B) return;
  const size_t row = (size_t)warp * A;
  float psum = 0.0f;
  for (int a0 = 0; a0 < A; a0 += kWarp) {
    const int a = a0 + lane;
    if (a < A) {
      const size_t i = row + a;
      const bool lg = legal[i] != 0;
      const bool cat = q_outcome[i] != -1;
      const float p = policy[i];
      psum += p;
      const float evidence_mass = visit[i];  // sum over the trailing singleton axis (+ 0)
      const bool positive_evidence = evidence_mass > 0.0f;
      const bool positive_policy = p > 0.0f;
      // _build_q_supervision (dirichlet_q_search.py:146-182)
      const bool source_selected = action_set == 0 ? positive_evidence : positive_policy;
      const float source_weight = action_set == 0 ? evidence_mass : p;
      const bool sel = lg && (source_selected || cat);
      float w;
      if (reduction == 0) {
        w = sel ? 1.0f : 0.0f;
      } else {
        // jnp.maximum(w, 1): a NaN weight stays NaN
        w = (lg && cat) ? (source_weight < 1.0f ? 1.0f : source_weight) : source_weight;
        w = sel ? w : 0.0f;
      }
      q_kind[i] = (int8_t)(lg ? (cat ? kTargetCategorical : kTargetDirichlet) : kTargetPad);
      selected[i] = sel;
      pair_weight[i] = w;
      pos_evidence[i] = lg && positive_evidence;
      pos_policy[i] = lg && positive_policy;
      q_weight[i] = lg ? 1.0f : 0.0f;
    }
  }
  // any order gives the same sign for a non-negative policy; a NaN keeps
  // the mask false as in the reference's sum
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) psum += __shfl_xor_sync(kFull, psum, off);
  if (lane == 0) {
    mask[warp] = psum > 0.0f;
    v_kind[warp] = (int8_t)(v_outcome[warp] != -1 ? kTargetCategorical : kTargetDirichlet);
    v_weight[warp] = 1.0f;
  }
}

// loss.py:511-517
__device__ __forceinline__ int outcome_index(float reward, int num_outcomes) {
  const int rounded = (int)rintf(reward);              // round half to even, as jnp.round
  return num_outcomes == 2 ? (rounded + 1) >> 1 : rounded + 1;  // floor division by 2
}

// One CTA per trajectory (lane b), threads over its T frames and then over
// its T x A (frame, action) cells.
__global__ void loss_input_kernel(scacchi_loss_frames f, scacchi_loss_out o, int B, int T, int A, int num_outcomes,
                                  int mask_mode, int winner_action, int terminal_edge, int terminal_parent,
                                  int legacy_reduction) {
  extern __shared__ float s_value[];  // [T] value targets, then [T] flags
  uint8_t *s_vmask = reinterpret_cast<uint8_t *>(s_value + T);
  const int b = blockIdx.x;
  const size_t f0 = (size_t)b * T;
  if (threadIdx.x == 0) {
    // loss.py:231-245: v_t = r_t + d_t * v_{t+1} from the end; the value
    // mask: a terminal frame at or after t inside the window
    float carry = 0.0f;
    int term_after = 0;
    for (int t = T - 1; t >= 0; --t) {
      const float prod = f.discount[f0 + t] * carry;
      carry = f.reward[f0 + t] + prod;
      s_value[t] = carry;
      term_after += f.terminated[f0 + t] != 0;
      s_vmask[t] = term_after >= 1;
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const size_t i = f0 + t;
    const float value_tgt = s_value[t];
    const bool value_mask = s_vmask[t] != 0;
    bool legal_any = false;
    float psum = 0.0f;
    for (int a = 0; a < A; ++a) {
      legal_any |= f.legal[i * A + a] != 0;
      psum += f.policy[i * A + a];
    }
    const bool search_loss = f.search_mask ? f.search_mask[i] != 0 : psum > 0.0f;
    bool policy_loss = legal_any && search_loss;
    bool value_loss = search_loss;
    if (mask_mode == 1) {  // value
      policy_loss = value_mask;
      value_loss = value_mask;
    } else if (mask_mode == 2) {  // pgx
      value_loss = value_mask;
    }
    if (winner_action) policy_loss = legal_any && value_mask && value_tgt > 0.0f;
    const bool terminated = f.terminated[i] != 0;
    const bool win = terminal_parent && terminated && f.reward[i] > 0.0f;
    if (win) {
      policy_loss = policy_loss || legal_any;
      value_loss = true;
    }
    o.value_tgt[i] = value_tgt;
    o.value_mask[i] = value_mask;
    o.policy_loss_mask[i] = policy_loss;
    o.value_loss_mask[i] = value_loss;
    o.search_loss_mask[i] = search_loss;
    // v sidecars: exact one-step outcome on a won terminal frame
    const int idx = outcome_index(f.reward[i], num_outcomes);
    o.v_kind[i] = win ? (int8_t)kTargetCategorical : f.v_kind[i];
    o.v_weight[i] = win ? 1.0f : f.v_weight[i];
    o.v_outcome[i] = win ? (int8_t)idx : f.v_outcome[i];
    o.v_distance[i] = win ? 1 : f.v_distance[i];
  }
  for (int c = threadIdx.x; c < T * A; c += blockDim.x) {
    const int t = c / A, a = c - t * A;
    const size_t i = f0 + t, j = i * A + a;
    const bool played = f.played_action[i] == a;
    const bool terminated = f.terminated[i] != 0;
    const bool win = terminal_parent && terminated && f.reward[i] > 0.0f;
    float p = winner_action ? (played ? 1.0f : 0.0f) : f.policy[j];
    if (win) p = played ? 1.0f : 0.0f;
    o.policy_tgt[j] = p;
    const bool edge = terminal_edge && terminated && played;
    const float w = f.q_pair_weight[j];
    o.q_pair_mask[j] = (f.q_pair_mask[j] != 0) || edge;
    // clamp(w, min=1): a NaN weight stays NaN
    o.q_pair_weight[j] = edge ? (legacy_reduction ? (w < 1.0f ? 1.0f : w) : 1.0f) : w;
    const int idx = outcome_index(f.reward[i], num_outcomes);
    o.q_kind[j] = edge ? (int8_t)kTargetCategorical : f.q_kind[j];
    o.q_weight[j] = edge ? 1.0f : f.q_weight[j];
    o.q_outcome[j] = edge ? (int8_t)idx : f.q_outcome[j];
    o.q_distance[j] = edge ? 1 : f.q_distance[j];
  }
}

bool al4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

extern "C" {

int scacchi_pack_targets(int32_t batch, int32_t num_actions, const float *visit_counts, const float *policy_target,
                         const uint8_t *legal, const int8_t *q_outcome, const int8_t *v_outcome, int32_t action_set,
                         int32_t reduction, int8_t *q_kind, int8_t *v_kind, uint8_t *mask, uint8_t *selected,
                         float *pair_weight, uint8_t *positive_evidence, uint8_t *positive_policy, float *q_weight,
                         float *v_weight, void *stream) {
  if (batch < 0 || num_actions < 1 || action_set < 0 || action_set > 1 || reduction < 0 || reduction > 1)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  if (!visit_counts || !policy_target || !legal || !q_outcome || !v_outcome || !q_kind || !v_kind || !mask ||
      !selected || !pair_weight || !positive_evidence || !positive_policy || !q_weight || !v_weight)
    return SCACCHI_EINVAL;
  if (!al4(visit_counts) || !al4(policy_target) || !al4(pair_weight) || !al4(q_weight) || !al4(v_weight))
    return SCACCHI_EINVAL;
  const int threads = 256, lanes_per_block = threads / kWarp;
  const int grid = (batch + lanes_per_block - 1) / lanes_per_block;
  pack_targets_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      batch, num_actions, visit_counts, policy_target, legal, q_outcome, v_outcome, action_set, reduction, q_kind,
      v_kind, mask, selected, pair_weight, positive_evidence, positive_policy, q_weight, v_weight);
  g_target_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaPeekAtLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

int scacchi_loss_input(const scacchi_loss_frames *frames, const scacchi_loss_out *out, int32_t batch,
                       int32_t frames_per_lane, int32_t num_actions, int32_t num_outcomes, int32_t loss_mask_mode,
                       int32_t winner_action_policy, int32_t terminal_edge_targets, int32_t terminal_parent_targets,
                       int32_t legacy_reduction, void *stream) {
  if (!frames || !out || batch < 0 || frames_per_lane < 1 || frames_per_lane > 4096 || num_actions < 1 ||
      (num_outcomes != 2 && num_outcomes != 3) || loss_mask_mode < 0 || loss_mask_mode > 2)
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  const scacchi_loss_frames &f = *frames;
  const scacchi_loss_out &o = *out;
  if (!f.reward || !f.discount || !f.terminated || !f.played_action || !f.legal || !f.policy || !f.q_pair_mask ||
      !f.q_pair_weight || !f.q_kind || !f.q_weight || !f.q_outcome || !f.q_distance || !f.v_kind || !f.v_weight ||
      !f.v_outcome || !f.v_distance)
    return SCACCHI_EINVAL;
  if (!o.value_tgt || !o.value_mask || !o.policy_loss_mask || !o.value_loss_mask || !o.search_loss_mask ||
      !o.policy_tgt || !o.q_pair_mask || !o.q_pair_weight || !o.q_kind || !o.q_weight || !o.q_outcome ||
      !o.q_distance || !o.v_kind || !o.v_weight || !o.v_outcome || !o.v_distance)
    return SCACCHI_EINVAL;
  const size_t smem = (size_t)frames_per_lane * (sizeof(float) + 1);
  loss_input_kernel<<<batch, 256, smem, static_cast<cudaStream_t>(stream)>>>(
      f, o, batch, frames_per_lane, num_actions, num_outcomes, loss_mask_mode, winner_action_policy != 0,
      terminal_edge_targets != 0, terminal_parent_targets != 0, legacy_reduction != 0);
  g_target_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaPeekAtLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

uint64_t scacchi_target_launch_count(void) { return g_target_launches.load(std::memory_order_relaxed); }

}  // extern "C"
