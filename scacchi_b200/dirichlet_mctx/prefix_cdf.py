"""Guardable binary posterior-best probabilities from prefix CDFs
(prefix_cdf.py of the reference), computed by the CUDA estimator kernel."""

from __future__ import annotations

import math
from typing import NamedTuple

import torch

from .. import _lib
from .outcomes import NO_OUTCOME
from .tree import ptr, stream_handle

MAX_HALF_WIDTH = 512


class BinaryPrefixQuadraturePolicy(NamedTuple):
    policy: torch.Tensor
    raw_policy: torch.Tensor
    raw_mass: torch.Tensor
    normalization_error: torch.Tensor
    finite: torch.Tensor
    grid_half_range: torch.Tensor
    tail_range_clipped: torch.Tensor
    density_log_integral: torch.Tensor
    fallback_interval_count: torch.Tensor


def validate_grid(half_width: int, tail_scale: float, min_half_range: float, max_half_range: float) -> None:
    """prefix_cdf.py:76-92, 271-272 (same messages)."""
    if not math.isfinite(tail_scale) or tail_scale <= 0.0:
        raise ValueError(f"tail_scale must be finite and > 0, got {tail_scale}")
    if not math.isfinite(min_half_range) or min_half_range <= 0.0:
        raise ValueError(f"min_half_range must be finite and > 0, got {min_half_range}")
    if not math.isfinite(max_half_range) or max_half_range < min_half_range:
        raise ValueError(
            f"max_half_range must be finite and >= min_half_range; got {max_half_range} and {min_half_range}")
    if half_width < 1:
        raise ValueError(f"half_width must be >= 1, got {half_width}")
    if half_width > MAX_HALF_WIDTH:
        raise ValueError(f"half_width must be <= {MAX_HALF_WIDTH} on this backend, got {half_width}")


def binary_posterior_best_policy_prefix_quadrature(
    alpha: torch.Tensor,
    invalid_actions: torch.Tensor,
    categorical_outcome: torch.Tensor | None = None,
    *,
    half_width: int = 10,
    tail_scale: float = 8.0,
    min_half_range: float = 6.0,
    max_half_range: float = 11.0,
) -> BinaryPrefixQuadraturePolicy:
    """prefix_cdf.py:217-445 on [B, A, 2] concentrations (leading axes other
    than one batch axis are flattened)."""
    if alpha.shape[-1] != 2:
        raise ValueError(f"binary prefix quadrature requires exactly two outcomes; got shape {tuple(alpha.shape)}")
    if tuple(invalid_actions.shape) != tuple(alpha.shape[:-1]):
        raise ValueError("invalid_actions must match alpha without its outcome axis; "
                         f"got {tuple(invalid_actions.shape)} and {tuple(alpha.shape)}")
    if categorical_outcome is not None and tuple(categorical_outcome.shape) != tuple(invalid_actions.shape):
        raise ValueError("categorical_outcome must match invalid_actions; "
                         f"got {tuple(categorical_outcome.shape)} and {tuple(invalid_actions.shape)}")
    validate_grid(half_width, tail_scale, min_half_range, max_half_range)
    lead = tuple(alpha.shape[:-2])
    A = alpha.shape[-2]
    B = int(math.prod(lead)) if lead else 1
    dev = alpha.device
    a = alpha.reshape(B, A, 2).to(torch.float32).contiguous()
    inv = invalid_actions.reshape(B, A).to(torch.uint8).contiguous()
    cat = None if categorical_outcome is None else categorical_outcome.reshape(B, A).to(torch.int8).contiguous()
    f32 = dict(dtype=torch.float32, device=dev)
    out = BinaryPrefixQuadraturePolicy(
        torch.empty((B, A), **f32), torch.empty((B, A), **f32), torch.empty((B,), **f32), torch.empty((B,), **f32),
        torch.empty((B,), dtype=torch.uint8, device=dev), torch.empty((B,), **f32),
        torch.empty((B,), dtype=torch.uint8, device=dev), torch.empty((B, A), **f32),
        torch.empty((B,), dtype=torch.int32, device=dev))
    po = _lib.PrefixOut(*[t.data_ptr() for t in out])
    _lib.check(_lib.lib().scacchi_prefix_cdf(ptr(a), ptr(inv), ptr(cat), B, A, int(half_width), float(tail_scale),
                                             float(min_half_range), float(max_half_range), po,
                                             stream_handle(dev)), "prefix_cdf")
    shaped = [t.reshape(*lead, *t.shape[1:]) for t in out]
    shaped[4] = shaped[4].bool()
    shaped[6] = shaped[6].bool()
    return BinaryPrefixQuadraturePolicy(*shaped)


__all__ = ["BinaryPrefixQuadraturePolicy", "binary_posterior_best_policy_prefix_quadrature", "NO_OUTCOME"]
