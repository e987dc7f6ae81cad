"""Contracts of the search (base.py of the reference), over torch tensors.

All tensors live on the CUDA device the search runs on.  Concentrations are
float32 with binary outcomes (loss, win).
"""

from __future__ import annotations

import dataclasses
from typing import Any, Callable, Generic, TypeVar

import torch

T = TypeVar("T")


@dataclasses.dataclass(frozen=True)
class RecurrentFnOutput:
    """base.py:58-74: the child's value prior [B, 2], action-value priors
    [B, A, 2], invalid actions [B, A], exact terminal outcome from the child's
    to_play perspective (or -1) [B] int8, and the child's to_play [B] int32."""

    value: torch.Tensor
    action_values: torch.Tensor
    invalid_actions: torch.Tensor
    terminal_outcome: torch.Tensor
    to_play: torch.Tensor


@dataclasses.dataclass(frozen=True)
class RootFnOutput:
    """base.py:80-93."""

    prior_logits: torch.Tensor
    value: torch.Tensor
    action_values: torch.Tensor
    embedding: Any
    terminal_outcome: torch.Tensor
    to_play: torch.Tensor


@dataclasses.dataclass(frozen=True)
class PolicyOutput(Generic[T]):
    """base.py:87-93: selected action, policy target and the finished tree."""

    action: torch.Tensor
    action_weights: torch.Tensor
    search_tree: T


RecurrentFn = Callable[[Any, Any, torch.Tensor, Any], tuple[RecurrentFnOutput, Any]]
