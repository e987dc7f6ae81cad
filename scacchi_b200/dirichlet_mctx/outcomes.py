"""Outcome sentinels and perspective helpers (outcomes.py of the reference).

Binary outcomes: index 0 = loss, 1 = win, from the node's player to move.
"""

from __future__ import annotations

import torch

NO_OUTCOME = -1
NO_DISTANCE = -1


def align_categorical_outcome(outcome: torch.Tensor, source_player: torch.Tensor, target_player: torch.Tensor,
                              num_outcomes: int = 2) -> torch.Tensor:
    """outcomes.py:21-27."""
    outcome = outcome.to(torch.int8)
    flipped = (num_outcomes - 1 - outcome).to(torch.int8)
    aligned = torch.where(source_player == target_player, outcome, flipped)
    return torch.where(outcome == NO_OUTCOME, torch.full_like(outcome, NO_OUTCOME), aligned)


def outcome_mean(alpha: torch.Tensor) -> torch.Tensor:
    return alpha / alpha.sum(-1, keepdim=True)


def outcome_utility(outcome: torch.Tensor) -> torch.Tensor:
    return outcome[..., -1] - outcome[..., 0]
