"""Loss-input assembly from self-play frames (scacchi/loss.py:30-55,
117-161, 164-357, 412-423, 511-517; native_targets.py).

``make_compute_input_for_lossfn(losses, num_outcomes)`` turns the
batch-major TrainingSamples of ``play.play_training`` into the ``Sample``
the losses read.  The frame-wise work -- trajectory value targets (a
reverse discounted scan), the value / policy / search loss masks of each
loss-mask mode, the winner-action policy target and the optional exact
one-step terminal targets -- is one CUDA kernel (scacchi_loss_input); this
module fills the sidecars a posterior without metadata lacks and binds the
kernel's outputs into the Sample.
"""

from __future__ import annotations

import ctypes as C
import dataclasses
from enum import StrEnum
from typing import NamedTuple

import torch

from . import _lib
from .dirichlet_mctx.outcomes import NO_OUTCOME
from .dirichlet_mctx.tree import ptr, stream_handle
from .play_search import TARGET_DIRICHLET
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


def _empty_posterior_targets(policy: torch.Tensor, num_outcomes: int):
    """loss.py:139-161."""
    q_pair_weight = policy * 0.0
    mask = torch.zeros_like(policy, dtype=torch.bool)
    beta_q = q_pair_weight[..., None].expand(*policy.shape, num_outcomes)
    beta_v = q_pair_weight.sum(-1, keepdim=True).expand(*policy.shape[:-1], num_outcomes)
    return beta_q, beta_v, mask, q_pair_weight


def make_compute_input_for_lossfn(losses: TrainingLossConfig, num_outcomes: int = 2):
    """loss.py:164-357 (frames on a CUDA device)."""
    mask_modes = {LossMaskMode.search: 0, LossMaskMode.value: 1, LossMaskMode.pgx: 2}

    def compute_loss_input(source) -> Sample:
        prediction = source.posterior.prediction
        metadata = source.posterior.metadata

        def metadata_value(field: str):
            return None if metadata is None else getattr(metadata, field, None)

        policy = prediction.policy
        if policy.device.type != "cuda":
            raise ValueError("the loss input is assembled on the GPU: pass frames on a CUDA device")
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
        native = _native_target_fields(metadata, beta_q, beta_v)
        B, T, A = policy.shape
        dev = policy.device
        # the terminal targets take the outcome count from beta_V (the
        # outcome index is only read with them; 2 stands in otherwise)
        terminal = losses.terminal_edge_targets or losses.terminal_parent_targets
        outcomes = beta_v.shape[-1] if terminal else 2
        if outcomes not in (2, 3):
            raise ValueError(f"unsupported outcome count: {outcomes}")

        def c(t, dtype):
            return t.to(device=dev, dtype=dtype).contiguous()

        f32, u8, i8, i32 = torch.float32, torch.uint8, torch.int8, torch.int32
        ins = dict(reward=c(source.reward, f32), discount=c(source.discount, f32),
                   terminated=c(source.terminated, u8), played_action=c(source.played_action, i32),
                   legal=c(source.legal_action_mask, u8), policy=c(policy, f32),
                   search_mask=None if metadata_value("mask") is None else c(metadata_value("mask"), u8),
                   q_pair_mask=c(q_pair_mask.expand(B, T, A), u8), q_pair_weight=c(q_pair_weight.expand(B, T, A), f32),
                   q_kind=c(native["q_target_kind"], i8), q_outcome=c(native["q_target_outcome"], i8),
                   q_weight=c(native["q_target_weight"], f32), q_distance=c(native["q_target_distance"], i32),
                   v_kind=c(native["v_target_kind"], i8), v_outcome=c(native["v_target_outcome"], i8),
                   v_weight=c(native["v_target_weight"], f32), v_distance=c(native["v_target_distance"], i32))
        outs = dict(value_tgt=torch.empty((B, T), dtype=f32, device=dev),
                    value_mask=torch.empty((B, T), dtype=u8, device=dev),
                    policy_loss_mask=torch.empty((B, T), dtype=u8, device=dev),
                    value_loss_mask=torch.empty((B, T), dtype=u8, device=dev),
                    search_loss_mask=torch.empty((B, T), dtype=u8, device=dev),
                    policy_tgt=torch.empty((B, T, A), dtype=f32, device=dev),
                    q_pair_mask=torch.empty((B, T, A), dtype=u8, device=dev),
                    q_pair_weight=torch.empty((B, T, A), dtype=f32, device=dev),
                    q_kind=torch.empty((B, T, A), dtype=i8, device=dev),
                    q_outcome=torch.empty((B, T, A), dtype=i8, device=dev),
                    q_weight=torch.empty((B, T, A), dtype=f32, device=dev),
                    q_distance=torch.empty((B, T, A), dtype=i32, device=dev),
                    v_kind=torch.empty((B, T), dtype=i8, device=dev), v_outcome=torch.empty((B, T), dtype=i8, device=dev),
                    v_weight=torch.empty((B, T), dtype=f32, device=dev),
                    v_distance=torch.empty((B, T), dtype=i32, device=dev))
        frames = _lib.LossFrames(*[ptr(ins[k]) for k in _lib.LossFrames.FIELDS])
        out = _lib.LossOut(*[ptr(outs[k]) for k in _lib.LossOut.FIELDS])
        legacy = losses.q_supervision.reduction == QPairReduction.legacy_normalized_source_weighted_mean
        _lib.check(_lib.lib().scacchi_loss_input(
            C.byref(frames), C.byref(out), B, T, A, outcomes, mask_modes[LossMaskMode(losses.loss_mask_mode)],
            int(PolicyTargetMode(losses.policy_target_mode) == PolicyTargetMode.winner_action),
            int(losses.terminal_edge_targets), int(losses.terminal_parent_targets), int(legacy),
            stream_handle(dev)), "loss_input")
        value_mask = outs["value_mask"].bool()
        return Sample(obs=source.obs, policy_tgt=outs["policy_tgt"], value_tgt=outs["value_tgt"],
                      played_action=source.played_action, policy_mask=source.legal_action_mask, value_mask=value_mask,
                      beta_Q_target=beta_q, beta_V_target=beta_v, q_supervised_pair_mask=outs["q_pair_mask"].bool(),
                      q_pair_weight=outs["q_pair_weight"], q_positive_evidence_action_mask=evidence,
                      q_positive_policy_action_mask=positive_policy,
                      policy_loss_mask=outs["policy_loss_mask"].bool(), value_loss_mask=outs["value_loss_mask"].bool(),
                      search_loss_mask=outs["search_loss_mask"].bool(), outcome_mask=value_mask,
                      q_target_kind=outs["q_kind"], q_target_weight=outs["q_weight"],
                      q_target_outcome=outs["q_outcome"], q_target_distance=outs["q_distance"],
                      v_target_kind=outs["v_kind"], v_target_weight=outs["v_weight"],
                      v_target_outcome=outs["v_outcome"], v_target_distance=outs["v_distance"])

    return compute_loss_input
