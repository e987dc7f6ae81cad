"""Public policy wrapper (policies.py of the reference)."""

from __future__ import annotations

from typing import Any, Callable

import numpy as np
import torch

from .. import _lib
from .. import random as srandom
from .base import PolicyOutput, RootFnOutput
from .posterior_updates import update_posterior
from .search import search
from .tree import Tree, ptr, stream_handle


def dirichlet_thompson_policy(params: Any, rng_key, *, root: RootFnOutput, recurrent_fn: Callable,
                              num_simulations: int, invalid_actions: torch.Tensor | None = None,
                              posterior_update: Callable = update_posterior, max_depth: int | None = None,
                              policy_samples: int = 32, policy_sample_chunk_size: int | None = None,
                              loop_fn: Callable | None = None,
                              stats: torch.Tensor | None = None) -> PolicyOutput[Tree]:
    """policies.py:17-48: search, then the root policy and its masked argmax."""
    if policy_samples < 0:
        raise ValueError(f"policy_samples must be >= 0, got {policy_samples}")
    if policy_sample_chunk_size is not None and policy_sample_chunk_size < 1:
        raise ValueError(f"chunk_size must be >= 1, got {policy_sample_chunk_size}")
    if invalid_actions is None:
        invalid_actions = ~torch.isfinite(root.prior_logits)
    keys = srandom.split(rng_key)
    search_key, policy_key = keys[0], keys[1]
    tree = search(params, search_key, root=root, recurrent_fn=recurrent_fn, posterior_update=posterior_update,
                  num_simulations=num_simulations, max_depth=max_depth, invalid_actions=invalid_actions,
                  stats=stats, loop_fn=loop_fn)
    dev = tree.device
    B, A = tree.batch, tree.A
    weights = torch.empty((B, A), dtype=torch.float32, device=dev)
    action = torch.empty((B,), dtype=torch.int32, device=dev)
    pk = torch.from_numpy(np.asarray(policy_key, np.uint32).view(np.int32).copy()).to(dev)
    inv = invalid_actions.to(device=dev, dtype=torch.uint8).contiguous()
    _lib.check(_lib.lib().scacchi_root_policy(tree.sref(), ptr(pk), ptr(inv), max(1, int(policy_samples)),
                                              ptr(weights), ptr(action), stream_handle(dev)), "root_policy")
    tree._keepalive_policy = (pk, inv)
    return PolicyOutput(action=action, action_weights=weights, search_tree=tree)
