"""The search()/evaluator boundary (scacchi/play_search.py of the reference).

``make_search(env, evaluator, search_cfg)`` returns
``search(root_state, rng_key) -> PosteriorTargets`` exactly like the
reference; the Dirichlet-Thompson search, its root readout and target packing
run on the GPU.  ``root_state`` follows the pgx.State fields the reference
reads: observation, legal_action_mask, current_player, rewards, terminated.

An env may provide ``native_recurrent_fn(evaluator)`` (a recurrent function
whose ``native_search`` runs the whole simulation loop in the CUDA library)
and ``embedding(root_state)`` (the per-node state record); otherwise the
generic expand function below calls ``env.step`` and ``evaluator`` from
Python once per simulation.
"""

from __future__ import annotations

import ctypes as C
import functools
from typing import Any, Callable, NamedTuple

import torch

from . import _lib
from .dirichlet_mctx import RecurrentFnOutput, RootFnOutput, dirichlet_thompson_policy
from .dirichlet_mctx.outcomes import NO_OUTCOME, align_categorical_outcome, outcome_mean, outcome_utility
from .dirichlet_mctx.posterior_updates import (DEFAULT_POLICY_SAMPLE_CHUNK_SIZE, update_posterior,
                                               update_posterior_prefix_cdf)
from .dirichlet_mctx.tree import ptr, stream_handle
from .types import (ActionCommitmentConfig, ActionCommitmentType, DirichletThompsonSearchConfig,
                    MonteCarloPosteriorUpdateConfig, NumericalPosteriorUpdateConfig, PosteriorUpdateKind, QActionSet,
                    QPairReduction, QSupervisionConfig, RootPolicySupport, SearchConfig, SearchKind)

TARGET_PAD = 0
TARGET_DIRICHLET = 1
TARGET_CATEGORICAL = 2


class EvaluatorOutput(NamedTuple):
    logits: torch.Tensor
    value: torch.Tensor | None = None
    alpha_v: torch.Tensor | None = None
    alpha_q: torch.Tensor | None = None


class PosteriorPrediction(NamedTuple):
    policy: torch.Tensor
    value: torch.Tensor | None = None
    alpha_v: torch.Tensor | None = None
    alpha_q: torch.Tensor | None = None


class QSupervision(NamedTuple):
    selected: torch.Tensor
    pair_weight: torch.Tensor


class TargetMetadata(NamedTuple):
    mask: torch.Tensor | None = None
    q_supervision: QSupervision | None = None
    q_positive_evidence_action: torch.Tensor | None = None
    q_positive_policy_action: torch.Tensor | None = None
    search_action: torch.Tensor | None = None
    q_target_kind: torch.Tensor | None = None
    q_target_weight: torch.Tensor | None = None
    q_target_outcome: torch.Tensor | None = None
    q_target_distance: torch.Tensor | None = None
    v_target_kind: torch.Tensor | None = None
    v_target_weight: torch.Tensor | None = None
    v_target_outcome: torch.Tensor | None = None
    v_target_distance: torch.Tensor | None = None


class PosteriorTargets(NamedTuple):
    prediction: PosteriorPrediction
    metadata: TargetMetadata | None = None


Search = Callable[[Any, Any], PosteriorTargets]


def evaluator_output_from_model_output(model_output: Any) -> EvaluatorOutput:
    """play_search.py:95-109."""
    if isinstance(model_output, EvaluatorOutput):
        return model_output
    if isinstance(model_output, torch.Tensor):
        return EvaluatorOutput(logits=model_output)
    logits, alpha_v, alpha_q = model_output
    return EvaluatorOutput(logits=logits, value=outcome_utility(outcome_mean(alpha_v)), alpha_v=alpha_v,
                           alpha_q=alpha_q)


def make_evaluator(model: Any) -> Callable[[torch.Tensor], EvaluatorOutput]:
    """play_search.py:112-118."""

    def evaluator(obs: torch.Tensor) -> EvaluatorOutput:
        return evaluator_output_from_model_output(model(obs))

    return evaluator


def _required_output(value, name: str):
    if value is None:
        raise ValueError(f"evaluator output is missing {name}")
    return value


def terminal_outcome_from_reward(reward: torch.Tensor, num_outcomes: int = 2) -> torch.Tensor:
    """dirichlet_q_search.py:27-40."""
    rounded = torch.round(reward).to(torch.int32)
    if num_outcomes == 2:
        outcome = torch.div(rounded + 1, 2, rounding_mode="floor")
    elif num_outcomes == 3:
        outcome = rounded + 1
    else:
        raise ValueError(f"unsupported outcome count: {num_outcomes}")
    return outcome.to(torch.int8)


def make_dirichlet_expand_fn(env: Any, evaluator: Callable):
    """dirichlet_q_search.py:43-76: env.step -> evaluator -> RecurrentFnOutput."""
    if hasattr(env, "native_recurrent_fn"):
        return env.native_recurrent_fn(evaluator)

    def expand_fn(_, rng_key, action: torch.Tensor, env_state: Any):
        del rng_key
        parent_player = env_state.current_player
        child = env.step(env_state, action)
        prediction = evaluator(child.observation)
        alpha_v = _required_output(prediction.alpha_v, "alpha_v")
        alpha_q = _required_output(prediction.alpha_q, "alpha_q")
        B = child.rewards.shape[0]
        reward = child.rewards[torch.arange(B, device=child.rewards.device), parent_player.long()]
        parent_outcome = terminal_outcome_from_reward(reward, alpha_v.shape[-1])
        child_outcome = align_categorical_outcome(parent_outcome, parent_player, child.current_player,
                                                  alpha_v.shape[-1])
        terminal = torch.where(child.terminated, child_outcome, torch.full_like(child_outcome, NO_OUTCOME))
        step = RecurrentFnOutput(value=alpha_v, action_values=alpha_q, invalid_actions=~child.legal_action_mask,
                                 terminal_outcome=terminal, to_play=child.current_player.to(torch.int32))
        return step, child

    return expand_fn


def _posterior_policy_sampling_budget(config) -> tuple[int, int]:
    """play_search.py:388-404."""
    if isinstance(config, NumericalPosteriorUpdateConfig):
        samples, chunk = config.fallback_policy_samples, config.fallback_policy_sample_chunk_size
    else:
        samples, chunk = config.policy_samples, config.policy_sample_chunk_size
    return int(samples), (max(1, int(chunk)) if chunk is not None else DEFAULT_POLICY_SAMPLE_CHUNK_SIZE)


def _make_posterior_update(config) -> Callable:
    """play_search.py:407-432."""
    samples, chunk = _posterior_policy_sampling_budget(config)
    if isinstance(config, NumericalPosteriorUpdateConfig):
        return functools.partial(update_posterior_prefix_cdf, kappa=float(config.kappa),
                                 half_width=int(config.half_width), tail_scale=float(config.tail_scale),
                                 min_half_range=float(config.min_half_range),
                                 max_half_range=float(config.max_half_range), fallback_policy_samples=samples,
                                 fallback_policy_sample_chunk_size=chunk)
    return functools.partial(update_posterior, kappa=float(config.kappa), policy_samples=samples,
                             policy_sample_chunk_size=chunk)


def build_q_supervision(action_set, reduction, q_search_count, posterior_policy_target, solved_action,
                        legal) -> QSupervision:
    """dirichlet_q_search.py:119-182."""
    evidence_mass = q_search_count.sum(-1) + torch.zeros_like(posterior_policy_target)
    positive_evidence = q_search_count.sum(-1) > 0
    positive_policy = posterior_policy_target > 0
    if action_set == QActionSet.positive_search_evidence_or_solved:
        source_selected, source_weight = positive_evidence, evidence_mass
    elif action_set == QActionSet.positive_posterior_policy_or_solved:
        source_selected, source_weight = positive_policy, posterior_policy_target
    else:
        raise ValueError(f"unknown Q action set: {action_set!r}")
    selected = legal & (source_selected | solved_action)
    if reduction == QPairReduction.mean_over_selected_state_action_pairs:
        pair_weight = selected.to(posterior_policy_target.dtype)
    elif reduction == QPairReduction.legacy_normalized_source_weighted_mean:
        pair_weight = torch.where(legal & solved_action, torch.clamp(source_weight, min=1.0), source_weight)
        pair_weight = torch.where(selected, pair_weight, torch.zeros_like(pair_weight))
    else:
        raise ValueError(f"unknown Q pair reduction: {reduction!r}")
    return QSupervision(selected=selected, pair_weight=pair_weight)


def dirichlet_root_policy_readout(native_policy: torch.Tensor, summary, legal_action_mask: torch.Tensor,
                                  search_cfg: DirichletThompsonSearchConfig) -> torch.Tensor:
    """play_search.py:298-364 (numerical update kind; the Monte Carlo kind
    returns the native policy unchanged)."""
    if search_cfg.posterior_update.kind != PosteriorUpdateKind.numerical:
        return native_policy
    num = search_cfg.posterior_update.numerical
    B, A = native_policy.shape
    dev = native_policy.device
    target = torch.empty((B, A), dtype=torch.float32, device=dev)
    legal = legal_action_mask.to(torch.uint8).contiguous()
    _lib.check(_lib.lib().scacchi_root_readout(
        B, A, ptr(native_policy.contiguous()), ptr(summary.visit_counts), ptr(summary.alpha),
        ptr(summary.q_categorical_outcome), ptr(summary.q_categorical_distance), ptr(summary.v_categorical_outcome),
        ptr(legal), int(search_cfg.root_policy_support == RootPolicySupport.search_evidence),
        float(search_cfg.policy_target_temperature), int(num.half_width), float(num.tail_scale),
        float(num.min_half_range), float(num.max_half_range), ptr(target), None, stream_handle(dev)),
        "root_readout")
    return target


def run_dirichlet_thompson_search(env_state, prediction: EvaluatorOutput, expand_fn, rng_key,
                                  search_cfg: DirichletThompsonSearchConfig,
                                  q_supervision_config: QSupervisionConfig, embedding: Any = None,
                                  stats: torch.Tensor | None = None, record: dict | None = None) -> PosteriorTargets:
    """play_search.py:435-548.  ``record``, when given, receives the search's
    PolicyOutput (tree included) under "policy_output"."""
    alpha_v = _required_output(prediction.alpha_v, "alpha_v")
    alpha_q = _required_output(prediction.alpha_q, "alpha_q")
    B = env_state.rewards.shape[0]
    dev = alpha_v.device
    player = env_state.current_player.long()
    root_reward = env_state.rewards[torch.arange(B, device=dev), player]
    root_terminal = torch.where(env_state.terminated, terminal_outcome_from_reward(root_reward, alpha_v.shape[-1]),
                                torch.full((B,), NO_OUTCOME, dtype=torch.int8, device=dev))
    root = RootFnOutput(prior_logits=prediction.logits, value=alpha_v, action_values=alpha_q,
                        embedding=env_state if embedding is None else embedding, terminal_outcome=root_terminal,
                        to_play=env_state.current_player.to(torch.int32))
    update_cfg = search_cfg.posterior_update.active()
    samples, chunk = _posterior_policy_sampling_budget(update_cfg)
    legal = env_state.legal_action_mask
    out = dirichlet_thompson_policy((), rng_key, root=root, recurrent_fn=expand_fn,
                                    num_simulations=int(search_cfg.num_simulations), invalid_actions=~legal,
                                    posterior_update=_make_posterior_update(update_cfg),
                                    max_depth=search_cfg.max_depth, policy_samples=samples,
                                    policy_sample_chunk_size=chunk, stats=stats)
    if record is not None:
        record["policy_output"] = out
    summary = out.search_tree.summary()
    policy_target = dirichlet_root_policy_readout(out.action_weights, summary, legal, search_cfg)
    metadata = pack_targets(summary, policy_target, legal, out.action, q_supervision_config)
    return PosteriorTargets(prediction=PosteriorPrediction(policy=policy_target, alpha_v=summary.value_alpha,
                                                           alpha_q=summary.alpha), metadata=metadata)


def pack_targets(summary, policy_target: torch.Tensor, legal: torch.Tensor, search_action: torch.Tensor,
                 q_supervision_config: QSupervisionConfig) -> TargetMetadata:
    """play_search.py:490-548 with build_q_supervision
    (dirichlet_q_search.py:119-182): the search's target metadata from the
    tree summary, in one kernel (scacchi_pack_targets).  beta_Q / beta_V,
    the categorical outcomes and distances are the summary's own tensors."""
    action_sets = {QActionSet.positive_search_evidence_or_solved: 0, QActionSet.positive_posterior_policy_or_solved: 1}
    reductions = {QPairReduction.mean_over_selected_state_action_pairs: 0,
                  QPairReduction.legacy_normalized_source_weighted_mean: 1}
    if q_supervision_config.action_set not in action_sets:
        raise ValueError(f"unknown Q action set: {q_supervision_config.action_set!r}")
    if q_supervision_config.reduction not in reductions:
        raise ValueError(f"unknown Q pair reduction: {q_supervision_config.reduction!r}")
    B, A = policy_target.shape
    dev = policy_target.device
    i8, u8, f32 = torch.int8, torch.uint8, torch.float32
    q_kind = torch.empty((B, A), dtype=i8, device=dev)
    v_kind = torch.empty((B,), dtype=i8, device=dev)
    mask = torch.empty((B,), dtype=u8, device=dev)
    selected = torch.empty((B, A), dtype=u8, device=dev)
    pair_weight = torch.empty((B, A), dtype=f32, device=dev)
    pos_evidence = torch.empty((B, A), dtype=u8, device=dev)
    pos_policy = torch.empty((B, A), dtype=u8, device=dev)
    q_weight = torch.empty((B, A), dtype=f32, device=dev)
    v_weight = torch.empty((B,), dtype=f32, device=dev)
    legal_u8 = legal.to(u8).contiguous()
    _lib.check(_lib.lib().scacchi_pack_targets(
        B, A, ptr(summary.visit_counts), ptr(policy_target.contiguous()), ptr(legal_u8),
        ptr(summary.q_categorical_outcome), ptr(summary.v_categorical_outcome),
        action_sets[q_supervision_config.action_set], reductions[q_supervision_config.reduction], ptr(q_kind),
        ptr(v_kind), ptr(mask), ptr(selected), ptr(pair_weight), ptr(pos_evidence), ptr(pos_policy), ptr(q_weight),
        ptr(v_weight), stream_handle(dev)), "pack_targets")
    return TargetMetadata(
        mask=mask.bool(), q_supervision=QSupervision(selected=selected.bool(), pair_weight=pair_weight),
        q_positive_evidence_action=pos_evidence.bool(), q_positive_policy_action=pos_policy.bool(),
        search_action=search_action, q_target_kind=q_kind, q_target_weight=q_weight,
        q_target_outcome=summary.q_categorical_outcome, q_target_distance=summary.q_categorical_distance,
        v_target_kind=v_kind, v_target_weight=v_weight, v_target_outcome=summary.v_categorical_outcome,
        v_target_distance=summary.v_categorical_distance)


def make_search(env, evaluator: Callable, search_cfg: SearchConfig | DirichletThompsonSearchConfig,
                q_supervision_config: QSupervisionConfig | None = None,
                stats: torch.Tensor | None = None, keep_output: bool = False) -> Search:
    """play_search.py:609-624 for the dirichlet_thompson kind.  With
    ``keep_output`` the returned function keeps its last call's PolicyOutput
    (action, action_weights, search_tree) in ``search.last_output`` for
    inspection; the tree then stays allocated until the next call."""
    if q_supervision_config is None:
        q_supervision_config = QSupervisionConfig()
    if isinstance(search_cfg, SearchConfig):
        if search_cfg.kind != SearchKind.dirichlet_thompson:
            raise ValueError(f"search kind {search_cfg.kind!s} is not implemented on this backend; "
                             "use dirichlet_thompson")
        search_cfg = search_cfg.dirichlet_thompson
    expand_fn = make_dirichlet_expand_fn(env, evaluator)
    embed = getattr(env, "embedding", None)

    def search(root_state, rng_key) -> PosteriorTargets:
        prediction = evaluator(root_state.observation)
        record = {} if keep_output else None
        targets = run_dirichlet_thompson_search(root_state, prediction, expand_fn, rng_key, search_cfg,
                                                q_supervision_config,
                                                embedding=embed(root_state) if embed is not None else None,
                                                stats=stats, record=record)
        if keep_output:
            search.last_output = record["policy_output"]
        return targets

    search.last_output = None
    return search


# --------------------------------------------------------------------------
# action commitment (play_search.py:627-831, dirichlet_q_search.py:79-116)
# --------------------------------------------------------------------------

def _commit(kind: int, rng_key, policy: torch.Tensor, legal_action_mask: torch.Tensor, temperature: float):
    from .dirichlet_mctx.action_selection import key_tensor

    B, A = policy.shape
    dev = policy.device
    action = torch.empty((B,), dtype=torch.int32, device=dev)
    key = key_tensor(rng_key, dev) if kind == 1 else None
    # converted operands stay referenced until the launch: a temporary freed
    # between two pointer grabs could hand its block to the next one
    pol = policy.to(torch.float32).contiguous()
    legal = legal_action_mask.to(torch.uint8).contiguous()
    _lib.check(_lib.lib().scacchi_commit_action(kind, ptr(key), ptr(pol), ptr(legal), B, A, float(temperature),
                                                ptr(action), stream_handle(dev)), "commit_action")
    return action


def posterior_best_action(policy_target: torch.Tensor, legal_action_mask: torch.Tensor) -> torch.Tensor:
    """dirichlet_q_search.py:79-86: argmax of the policy over legal actions."""
    return _commit(0, None, policy_target, legal_action_mask, 1.0)


def posterior_sample_action(rng_key, policy_target: torch.Tensor, legal_action_mask: torch.Tensor,
                            temperature: float = 1.0) -> torch.Tensor:
    """dirichlet_q_search.py:89-116: sample from the power-temperature
    transform of a root policy (jax.random.categorical on
    log(clip(p, 1e-8, 1)) / temperature over the legal actions with positive
    policy)."""
    import math

    if not math.isfinite(temperature) or temperature <= 0.0:
        raise ValueError(f"posterior sample temperature must be finite and > 0; got {temperature}.")
    return _commit(1, rng_key, policy_target, legal_action_mask, temperature)


def dirichlet_commitment_policy(posterior: PosteriorTargets, legal_action_mask: torch.Tensor, rng_key,
                                search_config: DirichletThompsonSearchConfig,
                                selected_update: PosteriorUpdateKind | None) -> torch.Tensor:
    """play_search.py:627-705: the root policy an action is committed from."""
    from .dirichlet_mctx.action_selection import posterior_best_policy

    prediction, metadata = posterior.prediction, posterior.metadata
    alpha = _required_output(prediction.alpha_q, "alpha_q")
    if (metadata is None or metadata.search_action is None or metadata.q_target_outcome is None
            or metadata.v_target_outcome is None):
        raise ValueError("Dirichlet action commitment requires root posterior metadata.")
    update_config = search_config.posterior_update.select(selected_update)
    samples, chunk = _posterior_policy_sampling_budget(update_config)
    dev = alpha.device
    legal = legal_action_mask.to(torch.bool)
    evidence = (torch.zeros_like(legal) if metadata.q_positive_evidence_action is None
                else metadata.q_positive_evidence_action.to(torch.bool))
    search_evidence = search_config.root_policy_support == RootPolicySupport.search_evidence
    candidate = legal & (evidence | (metadata.q_target_outcome != NO_OUTCOME))
    support = torch.where(candidate.any(-1, keepdim=True), candidate, legal) if search_evidence else legal
    # the full batch with the original key, as the reference samples it
    sampled = posterior_best_policy(rng_key, alpha, ~support, samples, chunk_size=chunk,
                                    categorical_outcome=metadata.q_target_outcome)
    B, A = sampled.shape
    numerical = isinstance(update_config, NumericalPosteriorUpdateConfig)
    num = search_config.posterior_update.numerical
    policy = torch.empty((B, A), dtype=torch.float32, device=dev)
    # converted operands stay referenced until the launch (see _commit)
    operands = (sampled.contiguous(), metadata.search_action.to(torch.int32).contiguous(), alpha.contiguous(),
                metadata.q_target_outcome.to(torch.int8).contiguous(),
                metadata.v_target_outcome.to(torch.int8).contiguous(), legal.to(torch.uint8).contiguous(),
                evidence.to(torch.uint8).contiguous())
    _lib.check(_lib.lib().scacchi_commitment_policy(
        B, A, *[ptr(t) for t in operands], int(search_evidence), int(numerical), int(num.half_width),
        float(num.tail_scale), float(num.min_half_range), float(num.max_half_range), ptr(policy),
        stream_handle(dev)), "commitment_policy")
    return policy


def make_action_committer(config: ActionCommitmentConfig,
                          dirichlet_search_config: DirichletThompsonSearchConfig | None = None) -> Callable:
    """play_search.py:708-750."""
    from . import random as srandom

    def action_committer(posterior: PosteriorTargets, legal_action_mask: torch.Tensor, rng_key) -> torch.Tensor:
        metadata = posterior.metadata
        search_action = None if metadata is None else metadata.search_action
        policy = posterior.prediction.policy
        action_key = rng_key
        if dirichlet_search_config is not None and config.kind != ActionCommitmentType.search_action:
            policy_key, action_key = srandom.split(rng_key)
            policy = dirichlet_commitment_policy(posterior, legal_action_mask, policy_key, dirichlet_search_config,
                                                 config.posterior_update)
        if config.kind == ActionCommitmentType.posterior_argmax:
            return posterior_best_action(policy, legal_action_mask)
        if config.kind == ActionCommitmentType.posterior_sample:
            return posterior_sample_action(action_key, policy, legal_action_mask,
                                           temperature=config.posterior_sample_temperature)
        if config.kind == ActionCommitmentType.search_action:
            if search_action is None:
                raise ValueError("search_action commitment requires a backend action")
            return search_action
        raise ValueError(f"unknown action_commitment_type: {config.kind!r}")

    return action_committer


def commit_action(action_commitment_type: str, rng_key, policy: torch.Tensor, legal_action_mask: torch.Tensor,
                  search_action: torch.Tensor | None = None, posterior_sample_temperature: float = 1.0):
    """play_search.py:753-784: commit an already-computed policy."""
    try:
        kind = ActionCommitmentType(action_commitment_type)
    except ValueError as error:
        raise ValueError(f"unknown action_commitment_type: {action_commitment_type!r}") from error
    posterior = PosteriorTargets(prediction=PosteriorPrediction(policy=policy),
                                 metadata=TargetMetadata(search_action=search_action))
    return make_action_committer(ActionCommitmentConfig(kind=kind,
                                                        posterior_sample_temperature=posterior_sample_temperature))(
        posterior, legal_action_mask, rng_key)


class PlayerOutput(NamedTuple):
    action: torch.Tensor
    posterior: PosteriorTargets


def make_search_player(env, model: Any, search_cfg: SearchConfig, action_commitment: ActionCommitmentConfig,
                       q_supervision_config: QSupervisionConfig | None = None) -> Callable:
    """play_search.py:799-831: search, then commit an action."""
    from . import random as srandom

    search = make_search(env, make_evaluator(model), search_cfg, q_supervision_config)
    committer = make_action_committer(
        action_commitment,
        search_cfg.dirichlet_thompson if search_cfg.kind == SearchKind.dirichlet_thompson else None)

    def player(env_state, rng_key) -> PlayerOutput:
        search_key, action_key = srandom.split(rng_key)
        posterior = search(env_state, search_key)
        action = committer(posterior, env_state.legal_action_mask, action_key)
        return PlayerOutput(action=action, posterior=posterior)

    return player
