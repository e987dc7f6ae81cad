"""CPU restatement of the loss-input assembly (scacchi/loss.py:30-55,
117-161, 164-357, 412-423, 511-517; native_targets.py) in torch tensor ops.

TEST INFRASTRUCTURE ONLY: the checker for scacchi_b200.loss_input (the
loss_input_kernel of csrc/targets.cu).  ``make_compute_input_for_lossfn``
turns batch-major TrainingSamples into the ``Sample`` the losses read: the
trajectory value targets (a reverse discounted scan), the value / policy /
search loss masks of each loss-mask mode, the winner-action policy target
and the optional exact one-step terminal targets.
"""

from __future__ import annotations

import torch

from scacchi_b200.loss_input import (LossMaskMode, PolicyTargetMode, Sample, TrainingLossConfig,
                                     _empty_posterior_targets, _native_target_fields)
from scacchi_b200.play_search import TARGET_CATEGORICAL
from scacchi_b200.types import QPairReduction


def _with_categorical_targets(targets: dict, head: str, mask: torch.Tensor, outcome: torch.Tensor) -> dict:
    """loss.py:117-136: exact one-step outcomes on the masked entries."""
    updated = dict(targets)
    for field, value in (("kind", TARGET_CATEGORICAL), ("weight", 1), ("outcome", outcome), ("distance", 1)):
        name = f"{head}_target_{field}"
        prev = updated[name]
        val = value if isinstance(value, torch.Tensor) else torch.tensor(value, device=prev.device)
        updated[name] = torch.where(mask, val.to(prev.dtype), prev)
    return updated


def _outcome_index(value_tgt: torch.Tensor, num_outcomes: int) -> torch.Tensor:
    """loss.py:511-517."""
    rounded = torch.round(value_tgt).to(torch.int32)
    if num_outcomes == 2:
        return torch.div(rounded + 1, 2, rounding_mode="floor")
    if num_outcomes == 3:
        return rounded + 1
    raise ValueError(f"unsupported outcome count: {num_outcomes}")


def trajectory_value_targets(reward: torch.Tensor, discount: torch.Tensor) -> torch.Tensor:
    """loss.py:231-245: v_t = r_t + d_t * v_{t+1}, scanned from the end of
    each [B, T] trajectory."""
    values = torch.empty_like(reward)
    carry = torch.zeros_like(reward[:, 0])
    for t in range(reward.shape[1] - 1, -1, -1):
        carry = reward[:, t] + discount[:, t] * carry
        values[:, t] = carry
    return values


def make_compute_input_for_lossfn(losses: TrainingLossConfig, num_outcomes: int = 2):
    """loss.py:164-357."""

    def compute_loss_input(source) -> Sample:
        prediction = source.posterior.prediction
        metadata = source.posterior.metadata

        def metadata_value(field: str):
            return None if metadata is None else getattr(metadata, field, None)

        policy = prediction.policy
        beta_q, beta_v = prediction.alpha_q, prediction.alpha_v
        q_supervision = metadata_value("q_supervision")
        if beta_q is None or beta_v is None or q_supervision is None:
            beta_q, beta_v, q_pair_mask, q_pair_weight = _empty_posterior_targets(policy, num_outcomes)
        else:
            q_pair_mask, q_pair_weight = q_supervision.selected, q_supervision.pair_weight
        evidence = metadata_value("q_positive_evidence_action")
        if evidence is None:
            evidence = torch.zeros_like(policy, dtype=torch.bool)
        positive_policy = metadata_value("q_positive_policy_action")
        if positive_policy is None:
            positive_policy = torch.zeros_like(policy, dtype=torch.bool)

        # a frame counts for the value once its trajectory ends inside the window
        value_mask = torch.flip(torch.cumsum(torch.flip(source.terminated.to(torch.int32), [1]), 1), [1]) >= 1
        legal_policy_mask = source.legal_action_mask.any(-1)
        metadata_mask = metadata_value("mask")
        search_loss_mask = metadata_mask if metadata_mask is not None else policy.sum(-1) > 0
        value_tgt = trajectory_value_targets(source.reward, source.discount)
        policy_tgt = policy
        policy_loss_mask = legal_policy_mask & search_loss_mask
        value_loss_mask = search_loss_mask
        mode = LossMaskMode(losses.loss_mask_mode)
        if mode == LossMaskMode.value:
            policy_loss_mask = value_mask
            value_loss_mask = value_mask
        elif mode == LossMaskMode.pgx:
            value_loss_mask = value_mask
        if PolicyTargetMode(losses.policy_target_mode) == PolicyTargetMode.winner_action:
            policy_tgt = torch.nn.functional.one_hot(source.played_action.long(), policy.shape[-1]).to(policy.dtype)
            policy_loss_mask = legal_policy_mask & value_mask & (value_tgt > 0)

        native = _native_target_fields(metadata, beta_q, beta_v)
        if losses.terminal_edge_targets or losses.terminal_parent_targets:
            outcome_index = _outcome_index(source.reward, beta_v.shape[-1])
            played = torch.nn.functional.one_hot(source.played_action.long(), beta_q.shape[-2]).to(torch.bool)
            terminal_action_mask = source.terminated[..., None] & played
        if losses.terminal_edge_targets:
            native = _with_categorical_targets(native, "q", terminal_action_mask, outcome_index[..., None])
            q_pair_mask = q_pair_mask | terminal_action_mask
            if losses.q_supervision.reduction == QPairReduction.legacy_normalized_source_weighted_mean:
                terminal_weight = torch.clamp(q_pair_weight, min=1.0)
            else:
                terminal_weight = torch.ones_like(q_pair_weight)
            q_pair_weight = torch.where(terminal_action_mask, terminal_weight, q_pair_weight)
        if losses.terminal_parent_targets:
            win = source.terminated & (source.reward > 0)
            policy_tgt = torch.where(win[..., None], played.to(policy_tgt.dtype), policy_tgt)
            policy_loss_mask = policy_loss_mask | (win & legal_policy_mask)
            value_loss_mask = value_loss_mask | win
            native = _with_categorical_targets(native, "v", win, outcome_index)

        return Sample(obs=source.obs, policy_tgt=policy_tgt, value_tgt=value_tgt, played_action=source.played_action,
                      policy_mask=source.legal_action_mask, value_mask=value_mask, beta_Q_target=beta_q,
                      beta_V_target=beta_v, q_supervised_pair_mask=q_pair_mask, q_pair_weight=q_pair_weight,
                      q_positive_evidence_action_mask=evidence, q_positive_policy_action_mask=positive_policy,
                      policy_loss_mask=policy_loss_mask, value_loss_mask=value_loss_mask,
                      search_loss_mask=search_loss_mask, outcome_mask=value_mask, **native)

    return compute_loss_input
