"""Bottom-up posterior repair rules (posterior_updates.py of the reference).

The two built-in rules are callable on an explicit PosteriorUpdateContext
(they then run the context kernel), and they are recognised by the search,
which runs the same rule fused into its backward kernel.  Callers configure
them exactly as in the reference, e.g.
``functools.partial(update_posterior_prefix_cdf, kappa=4.0, half_width=10)``.
Any other callable is rejected by the search: there is no host fallback.
"""

from __future__ import annotations

import functools
import math
from typing import Any, Callable

import numpy as np
import torch

from .. import _lib
from .action_selection import key_tensor
from .prefix_cdf import validate_grid
from .tree import PosteriorUpdate, PosteriorUpdateContext, ptr, stream_handle

DEFAULT_KAPPA = 4.0
DEFAULT_POLICY_SAMPLES = 32
DEFAULT_POLICY_SAMPLE_CHUNK_SIZE = 4
DEFAULT_PREFIX_DENSITY_LOG_INTEGRAL_TOLERANCE = 0.01


def _validate_kappa(kappa: float) -> None:
    if not math.isfinite(kappa) or kappa <= 0:
        raise ValueError(f"kappa must be finite and > 0, got {kappa}")


def _params(rule: int, kappa: float, samples: int, half_width: int = 10, tail_scale: float = 8.0,
            min_half_range: float = 6.0, max_half_range: float = 11.0,
            density_tol: float = DEFAULT_PREFIX_DENSITY_LOG_INTEGRAL_TOLERANCE) -> _lib.UpdateParams:
    return _lib.UpdateParams(
        rule, 1 if kappa >= 1.0 else 0, float(np.float32(1.0 / kappa)), float(np.float32(min(kappa, 1.0))), int(samples),
        int(half_width), float(tail_scale), float(min_half_range), float(max_half_range), float(density_tol))


def monte_carlo_params(*, kappa: float = DEFAULT_KAPPA, policy_samples: int = DEFAULT_POLICY_SAMPLES,
                       policy_sample_chunk_size: int = DEFAULT_POLICY_SAMPLE_CHUNK_SIZE) -> _lib.UpdateParams:
    """Validation of update_posterior (posterior_updates.py:335-349)."""
    _validate_kappa(kappa)
    if policy_samples < 1:
        raise ValueError(f"policy_samples must be >= 1, got {policy_samples}")
    if policy_sample_chunk_size < 1:
        raise ValueError(f"policy_sample_chunk_size must be >= 1, got {policy_sample_chunk_size}")
    return _params(0, kappa, policy_samples)


def prefix_cdf_params(*, kappa: float = DEFAULT_KAPPA, half_width: int = 10, tail_scale: float = 8.0,
                      min_half_range: float = 6.0, max_half_range: float = 11.0,
                      fallback_policy_samples: int = DEFAULT_POLICY_SAMPLES,
                      fallback_policy_sample_chunk_size: int = DEFAULT_POLICY_SAMPLE_CHUNK_SIZE,
                      density_log_integral_tolerance: float = DEFAULT_PREFIX_DENSITY_LOG_INTEGRAL_TOLERANCE,
                      ) -> _lib.UpdateParams:
    """Validation of update_posterior_prefix_cdf (posterior_updates.py:247-270)."""
    _validate_kappa(kappa)
    if fallback_policy_samples < 1:
        raise ValueError(f"fallback_policy_samples must be >= 1, got {fallback_policy_samples}")
    if fallback_policy_sample_chunk_size < 1:
        raise ValueError(
            f"fallback_policy_sample_chunk_size must be >= 1, got {fallback_policy_sample_chunk_size}")
    if not math.isfinite(density_log_integral_tolerance) or density_log_integral_tolerance <= 0.0:
        raise ValueError(
            f"density_log_integral_tolerance must be finite and > 0, got {density_log_integral_tolerance}")
    validate_grid(half_width, tail_scale, min_half_range, max_half_range)
    return _params(1, kappa, fallback_policy_samples, half_width, tail_scale, min_half_range, max_half_range,
                   density_log_integral_tolerance)


def _run_context(rng_key, context: PosteriorUpdateContext, params: _lib.UpdateParams) -> PosteriorUpdate:
    node, children, leaf = context.node, context.children, context.leaf
    if node.edge_alpha.shape[-1] != 2:
        raise ValueError("prefix-CDF posterior repair requires exactly two outcomes; "
                         f"got {node.edge_alpha.shape[-1]}")
    B, A, _ = node.edge_alpha.shape
    dev = node.edge_alpha.device

    def c(t, dt):
        return torch.as_tensor(t).to(device=dev, dtype=dt).contiguous()

    f, i32, i8, u8 = torch.float32, torch.int32, torch.int8, torch.uint8
    fields = [
        c(context.active, u8), c(leaf.active, u8), c(leaf.action, i32), c(leaf.value_alpha, f),
        c(leaf.to_play, i32), c(node.to_play, i32), c(node.node_payload, i32), c(node.value_prior, f),
        c(node.value_alpha, f), c(node.edge_alpha, f), c(node.edge_payload, i32),
        c(node.edge_categorical_outcome, i8), c(node.invalid_actions, u8), c(children.visited, u8),
        c(children.value_prior, f), c(children.value_alpha, f), c(children.node_payload, i32),
        c(children.categorical_outcome, i8), c(children.to_play, i32)]
    ctx = _lib.Context(*[t.data_ptr() for t in fields])
    ea = torch.empty((B, A, 2), dtype=f, device=dev)
    ep = torch.empty((B, A), dtype=i32, device=dev)
    va = torch.empty((B, 2), dtype=f, device=dev)
    unsafe = torch.empty((B,), dtype=u8, device=dev)
    k = key_tensor(rng_key, dev)
    _lib.check(_lib.lib().scacchi_update_posterior(ptr(k), ctx, B, A, params, ptr(ea), ptr(ep), ptr(va),
                                                   ptr(unsafe), stream_handle(dev)), "update_posterior")
    return PosteriorUpdate(edge_alpha=ea, edge_payload=ep, value_alpha=va)


def update_posterior(rng_key, context: PosteriorUpdateContext, *, kappa: float = DEFAULT_KAPPA,
                     policy_samples: int = DEFAULT_POLICY_SAMPLES,
                     policy_sample_chunk_size: int = DEFAULT_POLICY_SAMPLE_CHUNK_SIZE) -> PosteriorUpdate:
    """posterior_updates.py:335-367 (Monte Carlo winner population)."""
    return _run_context(rng_key, context, monte_carlo_params(
        kappa=kappa, policy_samples=policy_samples, policy_sample_chunk_size=policy_sample_chunk_size))


def update_posterior_prefix_cdf(rng_key, context: PosteriorUpdateContext, *, kappa: float = DEFAULT_KAPPA,
                                half_width: int = 10, tail_scale: float = 8.0, min_half_range: float = 6.0,
                                max_half_range: float = 11.0, fallback_policy_samples: int = DEFAULT_POLICY_SAMPLES,
                                fallback_policy_sample_chunk_size: int = DEFAULT_POLICY_SAMPLE_CHUNK_SIZE,
                                density_log_integral_tolerance: float =
                                DEFAULT_PREFIX_DENSITY_LOG_INTEGRAL_TOLERANCE) -> PosteriorUpdate:
    """posterior_updates.py:220-332 (guarded prefix-CDF Q21 with the per-lane
    Monte Carlo fallback)."""
    if context.node.edge_alpha.shape[-1] != 2:
        raise ValueError("prefix-CDF posterior repair requires exactly two outcomes; "
                         f"got {context.node.edge_alpha.shape[-1]}")
    return _run_context(rng_key, context, prefix_cdf_params(
        kappa=kappa, half_width=half_width, tail_scale=tail_scale, min_half_range=min_half_range,
        max_half_range=max_half_range, fallback_policy_samples=fallback_policy_samples,
        fallback_policy_sample_chunk_size=fallback_policy_sample_chunk_size,
        density_log_integral_tolerance=density_log_integral_tolerance))


def rule_params(posterior_update: Callable[..., Any]) -> _lib.UpdateParams:
    """Static parameters of a built-in rule or a functools.partial of one."""
    fn, kw = posterior_update, {}
    while isinstance(fn, functools.partial):
        if fn.args:
            raise ValueError("posterior_update partials may only bind keyword arguments")
        kw = {**fn.keywords, **kw}
        fn = fn.func
    if fn is update_posterior:
        return monte_carlo_params(**kw)
    if fn is update_posterior_prefix_cdf:
        return prefix_cdf_params(**kw)
    raise ValueError("the native search runs update_posterior or update_posterior_prefix_cdf "
                     f"(optionally through functools.partial); got {posterior_update!r}")
