"""Search configuration (the search-step part of scacchi/types.py).

Same field names, defaults and validation messages as the reference's
dataclasses (types.py:24-28, 170-345, 362-377, 394-400).  Only the Dirichlet-Thompson search
runs on this backend; the policy and Gumbel search kinds are accepted as
configuration but rejected by ``make_search``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from enum import StrEnum


class ActionCommitmentType(StrEnum):
    posterior_argmax = "posterior_argmax"
    posterior_sample = "posterior_sample"
    search_action = "search_action"


class SearchKind(StrEnum):
    policy = "policy"
    gumbel = "gumbel"
    dirichlet_thompson = "dirichlet_thompson"


class PosteriorUpdateKind(StrEnum):
    monte_carlo = "monte_carlo"
    numerical = "numerical"


class RootPolicySupport(StrEnum):
    all_legal = "all_legal"
    search_evidence = "search_evidence"


class QActionSet(StrEnum):
    positive_search_evidence_or_solved = "positive_search_evidence_or_solved"
    positive_posterior_policy_or_solved = "positive_posterior_policy_or_solved"


class QPairReduction(StrEnum):
    mean_over_selected_state_action_pairs = "mean_over_selected_state_action_pairs"
    legacy_normalized_source_weighted_mean = "legacy_normalized_source_weighted_mean"


def _require_ge(name: str, value, minimum) -> None:
    if value is not None and value < minimum:
        raise ValueError(f"{name} must be >= {minimum}; got {value}.")


def _require_gt(name: str, value, minimum: float) -> None:
    if value is not None and (not math.isfinite(float(value)) or value <= minimum):
        raise ValueError(f"{name} must be > {minimum}; got {value}.")


@dataclass
class PolicySearchConfig:
    temperature: float = 1.0

    def __post_init__(self) -> None:
        _require_gt("search.policy.temperature", self.temperature, 0.0)


@dataclass
class GumbelSearchConfig:
    num_simulations: int = 32
    gumbel_scale: float = 1.0

    def __post_init__(self) -> None:
        _require_ge("search.gumbel.num_simulations", self.num_simulations, 1)
        _require_gt("search.gumbel.gumbel_scale", self.gumbel_scale, 0.0)


@dataclass
class MonteCarloPosteriorUpdateConfig:
    kappa: float = 4.0
    policy_samples: int = 32
    policy_sample_chunk_size: int | None = 32

    def __post_init__(self) -> None:
        if not math.isfinite(self.kappa):
            raise ValueError("search.dirichlet_thompson.posterior_update.monte_carlo.kappa "
                             f"must be finite; got {self.kappa}.")
        _require_gt("search.dirichlet_thompson.posterior_update.monte_carlo.kappa", self.kappa, 0.0)
        _require_ge("search.dirichlet_thompson.posterior_update.monte_carlo.policy_samples",
                    self.policy_samples, 1)
        _require_ge("search.dirichlet_thompson.posterior_update.monte_carlo.policy_sample_chunk_size",
                    self.policy_sample_chunk_size, 1)


@dataclass
class NumericalPosteriorUpdateConfig:
    kappa: float = 4.0
    half_width: int = 10
    tail_scale: float = 8.0
    min_half_range: float = 6.0
    max_half_range: float = 11.0
    fallback_policy_samples: int = 32
    fallback_policy_sample_chunk_size: int | None = 32

    def __post_init__(self) -> None:
        if not math.isfinite(self.kappa):
            raise ValueError("search.dirichlet_thompson.posterior_update.numerical.kappa "
                             f"must be finite; got {self.kappa}.")
        _require_gt("search.dirichlet_thompson.posterior_update.numerical.kappa", self.kappa, 0.0)
        _require_ge("search.dirichlet_thompson.posterior_update.numerical.fallback_policy_samples",
                    self.fallback_policy_samples, 1)
        _require_ge("search.dirichlet_thompson.posterior_update.numerical.fallback_policy_sample_chunk_size",
                    self.fallback_policy_sample_chunk_size, 1)
        _require_ge("search.dirichlet_thompson.posterior_update.numerical.half_width", self.half_width, 1)
        for name, value in (("search.dirichlet_thompson.posterior_update.numerical.tail_scale", self.tail_scale),
                            ("search.dirichlet_thompson.posterior_update.numerical.min_half_range",
                             self.min_half_range)):
            if not math.isfinite(value) or value <= 0.0:
                raise ValueError(f"{name} must be finite and > 0; got {value}.")
        if not math.isfinite(self.max_half_range) or self.max_half_range < self.min_half_range:
            raise ValueError("search.dirichlet_thompson.posterior_update.numerical.max_half_range must be finite "
                             f"and >= min_half_range; got {self.max_half_range} and {self.min_half_range}.")


@dataclass
class PosteriorUpdateConfig:
    kind: PosteriorUpdateKind = PosteriorUpdateKind.monte_carlo
    monte_carlo: MonteCarloPosteriorUpdateConfig = field(default_factory=MonteCarloPosteriorUpdateConfig)
    numerical: NumericalPosteriorUpdateConfig = field(default_factory=NumericalPosteriorUpdateConfig)

    def select(self, kind: PosteriorUpdateKind | None = None):
        return getattr(self, str(self.kind if kind is None else kind))

    def active(self):
        return self.select()


@dataclass
class DirichletThompsonSearchConfig:
    num_simulations: int = 32
    max_depth: int | None = None
    root_policy_support: RootPolicySupport = RootPolicySupport.all_legal
    policy_target_temperature: float = 1.0
    posterior_update: PosteriorUpdateConfig = field(default_factory=PosteriorUpdateConfig)

    def __post_init__(self) -> None:
        _require_ge("search.dirichlet_thompson.num_simulations", self.num_simulations, 0)
        if self.max_depth is None:
            self.max_depth = self.num_simulations
        _require_ge("search.dirichlet_thompson.max_depth", self.max_depth, 1 if self.num_simulations > 0 else 0)
        if not math.isfinite(self.policy_target_temperature) or self.policy_target_temperature <= 0.0:
            raise ValueError("search.dirichlet_thompson.policy_target_temperature must be finite and > 0; got "
                             f"{self.policy_target_temperature}.")


@dataclass
class SearchConfig:
    kind: SearchKind = SearchKind.gumbel
    policy: PolicySearchConfig = field(default_factory=PolicySearchConfig)
    gumbel: GumbelSearchConfig = field(default_factory=GumbelSearchConfig)
    dirichlet_thompson: DirichletThompsonSearchConfig = field(default_factory=DirichletThompsonSearchConfig)

    def active(self):
        return getattr(self, str(self.kind))


@dataclass
class QSupervisionConfig:
    action_set: QActionSet = QActionSet.positive_search_evidence_or_solved
    reduction: QPairReduction = QPairReduction.mean_over_selected_state_action_pairs


@dataclass
class ActionCommitmentConfig:
    """types.py:362-377 of the reference."""

    kind: ActionCommitmentType = ActionCommitmentType.posterior_argmax
    # None reuses the updater selected by Dirichlet Thompson search.
    posterior_update: PosteriorUpdateKind | None = None
    posterior_sample_temperature: float = 1.0

    def __post_init__(self) -> None:
        if not math.isfinite(self.posterior_sample_temperature) or self.posterior_sample_temperature <= 0.0:
            raise ValueError("action_commitment.posterior_sample_temperature must be finite and > 0; got "
                             f"{self.posterior_sample_temperature}.")
