"""Run a ``tests/scenarios.py`` scenario on the C oracle."""

from __future__ import annotations

import types

import numpy as np

from oracle import oracle as O


def run(sc, rule=None):
    if rule is None:
        rule = O.Rule(prefix_cdf=sc.prefix_cdf, samples=32, kappa=4.0)
    root = dict(sc.root)
    root["embedding"] = np.ascontiguousarray(root["embedding"], np.int32).view(np.uint8).reshape(-1, 4)

    def recurrent(action, parent_emb):
        depth = np.ascontiguousarray(parent_emb).view(np.int32).reshape(-1)
        step, child = sc.step(action, depth)
        return step, np.ascontiguousarray(child, np.int32).view(np.uint8).reshape(-1, 4)

    out = O.dirichlet_thompson_policy(
        sc.rng_key, root=root, recurrent_fn=recurrent, num_simulations=sc.num_simulations,
        invalid_actions=sc.invalid_actions if sc.invalid_actions is not None else np.zeros_like(
            root["prior_logits"], bool),
        rule=rule, max_depth=sc.max_depth, policy_samples=sc.policy_samples)
    return types.SimpleNamespace(tree=out.search_tree, action=out.action, action_weights=out.action_weights)
