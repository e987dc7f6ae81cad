"""Loss-input assembly from self-play frames (scacchi/loss.py:30-55,
117-161, 164-357, 412-423, 511-517; native_targets.py).

``make_compute_input_for_lossfn(losses, num_outcomes)`` turns the
batch-major TrainingSamples of ``play.play_training`` into the ``Sample``
the losses read: trajectory value targets (a reverse discounted scan),
the value/policy/search loss masks of each loss-mask mode, the winner-action
policy target, and the optional exact one-step terminal targets, all as
device tensor operations.
"""

from __future__ import annotations

import dataclasses
from enum import StrEnum
from typing import NamedTuple

import torch

from .dirichlet_mctx.outcomes import NO_OUTCOME
from .play_search import TARGET_CATEGORICAL, TARGET_DIRICHLET
from .types import QPairReduction, QSupervisionConfig

NO_DISTANCE = -1


class LossMaskMode(StrEnum):
    search = "search"
    value = "value"
    pgx = "pgx"


class PolicyTargetMode(StrEnum):
    search = "search"
    winner_action = "winner_action"


@dataclasses.dataclass
class TrainingLossConfig:
    """The fields of types.py:403-419 the loss input reads."""

    q_supervision: QSupervisionConfig = dataclasses.field(default_factory=QSupervisionConfig)
    loss_mask_mode: LossMaskMode = LossMaskMode.search
    terminal_edge_targets: bool = False
    terminal_parent_targets: bool = False
    policy_target_mode: PolicyTargetMode = PolicyTargetMode.search


class Sample(NamedTuple):
    """loss.py:30-55."""

    obs: torch.Tensor
    policy_tgt: torch.Tensor
    value_tgt: torch.Tensor
    played_action: torch.Tensor
    policy_mask: torch.Tensor
    value_mask: torch.Tensor
    beta_Q_target: torch.Tensor
    beta_V_target: torch.Tensor
    q_supervised_pair_mask: torch.Tensor
    q_pair_weight: torch.Tensor
    q_positive_evidence_action_mask: torch.Tensor | None = None
    q_positive_policy_action_mask: torch.Tensor | None = None
    policy_loss_mask: torch.Tensor | None = None
    value_loss_mask: torch.Tensor | None = None
    search_loss_mask: torch.Tensor | None = None
    outcome_mask: torch.Tensor | None = None
    q_target_kind: torch.Tensor | None = None
    q_target_weight: torch.Tensor | None = None
    q_target_outcome: torch.Tensor | None = None
    q_target_distance: torch.Tensor | None = None
    v_target_kind: torch.Tensor | None = None
    v_target_weight: torch.Tensor | None = None
    v_target_outcome: torch.Tensor | None = None
    v_target_distance: torch.Tensor | None = None


NATIVE_FIELDS = ("q_target_kind", "q_target_weight", "q_target_outcome", "q_target_distance", "v_target_kind",
                 "v_target_weight", "v_target_outcome", "v_target_distance")


def native_fields_from_beta(beta_q: torch.Tensor, beta_v: torch.Tensor) -> dict:
    """native_targets.py:45-60: ordinary-Dirichlet sidecars."""
    out = {}
    for head, beta in (("q", beta_q), ("v", beta_v)):
        t = beta[..., 0]
        out[f"{head}_target_kind"] = torch.full_like(t, TARGET_DIRICHLET, dtype=torch.int8)
        out[f"{head}_target_weight"] = torch.ones_like(t)
        out[f"{head}_target_outcome"] = torch.full_like(t, NO_OUTCOME, dtype=torch.int8)
        out[f"{head}_target_distance"] = torch.full_like(t, NO_DISTANCE, dtype=torch.int32)
    return out


def _native_target_fields(metadata, beta_q, beta_v) -> dict:
    """loss.py:412-423: fill missing sidecars, keep complete ones."""
    values = {f: (None if metadata is None else getattr(metadata, f, None)) for f in NATIVE_FIELDS}
    if any(v is None for v in values.values()):
        defaults = native_fields_from_beta(beta_q, beta_v)
        values = {f: defaults[f] if values[f] is None else values[f] for f in NATIVE_FIELDS}
    return values


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


def _empty_posterior_targets(policy: torch.Tensor, num_outcomes: int):
    """loss.py:139-161."""
    q_pair_weight = policy * 0.0
    mask = torch.zeros_like(policy, dtype=torch.bool)
    beta_q = q_pair_weight[..., None].expand(*policy.shape, num_outcomes)
    beta_v = q_pair_weight.sum(-1, keepdim=True).expand(*policy.shape[:-1], num_outcomes)
    return beta_q, beta_v, mask, q_pair_weight


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
