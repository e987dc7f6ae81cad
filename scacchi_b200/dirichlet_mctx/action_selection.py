"""Thompson action selection (action_selection.py of the reference)."""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from .. import _lib
from .outcomes import NO_OUTCOME
from .tree import ptr, stream_handle


def key_tensor(key, device) -> torch.Tensor:
    k = np.asarray(key, dtype=np.uint32).reshape(2)
    return torch.from_numpy(k.view(np.int32).copy()).to(device)


def _common(alpha, invalid_actions, categorical_outcome):
    if alpha.dim() != 3 or alpha.shape[-1] != 2:
        raise ValueError(f"alpha must be [batch, action, 2], got {tuple(alpha.shape)}")
    B, A, _ = alpha.shape
    dev = alpha.device
    a = alpha.to(torch.float32).contiguous()
    inv = invalid_actions.to(device=dev, dtype=torch.uint8).contiguous()
    cat = None if categorical_outcome is None else categorical_outcome.to(device=dev, dtype=torch.int8).contiguous()
    return B, A, dev, a, inv, cat


def posterior_best_policy(rng_key, alpha: torch.Tensor, invalid_actions: torch.Tensor, num_samples: int, *,
                          chunk_size: int | None = None,
                          categorical_outcome: torch.Tensor | None = None) -> torch.Tensor:
    """action_selection.py:146-194.  ``chunk_size`` only bounds memory in the
    reference and does not change the result; it is validated and ignored."""
    if num_samples < 1:
        raise ValueError(f"num_samples must be >= 1, got {num_samples}")
    if chunk_size is not None and chunk_size < 1:
        raise ValueError(f"chunk_size must be >= 1, got {chunk_size}")
    B, A, dev, a, inv, cat = _common(alpha, invalid_actions, categorical_outcome)
    out = torch.empty((B, A), dtype=torch.float32, device=dev)
    k = key_tensor(rng_key, dev)
    _lib.check(_lib.lib().scacchi_posterior_best_policy(ptr(k), ptr(a), ptr(inv), ptr(cat), B, A, int(num_samples),
                                                        ptr(out), stream_handle(dev)), "posterior_best_policy")
    return out


def thompson_sample(rng_key, alpha: torch.Tensor, invalid_actions: torch.Tensor,
                    categorical_outcome: torch.Tensor | None = None) -> torch.Tensor:
    """action_selection.py:135-143."""
    B, A, dev, a, inv, cat = _common(alpha, invalid_actions, categorical_outcome)
    out = torch.empty((B,), dtype=torch.int32, device=dev)
    k = key_tensor(rng_key, dev)
    _lib.check(_lib.lib().scacchi_thompson_sample(ptr(k), ptr(a), ptr(inv), ptr(cat), B, A, ptr(out),
                                                  stream_handle(dev)), "thompson_sample")
    return out


def masked_argmax(scores: torch.Tensor, invalid_actions: torch.Tensor) -> torch.Tensor:
    """action_selection.py:78-79."""
    return torch.argmax(torch.where(invalid_actions, torch.full_like(scores, -float("inf")), scores), dim=-1).to(
        torch.int32)


def categorical_action_population(node_outcome, edge_outcome, edge_distance, invalid_actions, *,
                                  num_outcomes: int = 2, dtype=torch.float32) -> torch.Tensor:
    """action_selection.py:24-49, 62-75 (binary outcomes)."""
    legal = ~invalid_actions
    dist = edge_distance.to(torch.float32)
    ninf = torch.full_like(dist, -float("inf"))
    win = torch.where(legal & (edge_outcome == 1), -dist, ninf)
    loss = torch.where(legal & (edge_outcome == 0), dist, ninf)
    draw = torch.where(legal & (edge_outcome == 1), torch.zeros_like(dist), ninf)
    no = node_outcome[..., None]
    scores = torch.where(no == 1, win, torch.where(no == 0, loss, draw))
    best = scores.max(dim=-1, keepdim=True).values
    tied = torch.isfinite(scores) & (scores == best)
    count = tied.sum(-1, keepdim=True)
    return tied.to(dtype) / torch.clamp(count, min=1).to(dtype)


__all__ = ["posterior_best_policy", "thompson_sample", "masked_argmax", "categorical_action_population",
           "NO_OUTCOME"]
