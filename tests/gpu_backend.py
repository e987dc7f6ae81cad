"""Run a ``tests/scenarios.py`` scenario through the CUDA search and return a
numpy view with the oracle's field names."""

from __future__ import annotations

import types

import numpy as np
import torch

from scacchi_b200 import dirichlet_mctx as dm
from scacchi_b200.dirichlet_mctx.posterior_updates import update_posterior, update_posterior_prefix_cdf
import functools


class NumpyTree:
    """Host copy of a device Tree with the reference's field names."""

    def __init__(self, tree):
        for name in ("parents", "children_index", "node_to_play", "node_categorical_outcome", "node_payload",
                     "edge_categorical_outcome", "edge_payload", "node_value_priors", "node_value_alpha",
                     "edge_alpha"):
            setattr(self, name, getattr(tree, name).cpu().numpy())
        self.invalid_actions = tree.invalid_actions.cpu().numpy().astype(np.uint8)
        self._summary = {k: v.cpu().numpy() for k, v in vars(tree.summary()).items()}

    def summary(self):
        return self._summary


def run(sc, device="cuda", kappa=4.0, samples=32):
    dev = torch.device(device)
    r = sc.root
    t = lambda x, dt: torch.as_tensor(np.asarray(x)).to(dev, dt)
    root = dm.RootFnOutput(prior_logits=t(r["prior_logits"], torch.float32), value=t(r["value"], torch.float32),
                           action_values=t(r["action_values"], torch.float32),
                           embedding=t(r["embedding"], torch.int32),
                           terminal_outcome=t(r["terminal_outcome"], torch.int8),
                           to_play=t(r["to_play"], torch.int32))

    def recurrent(params, key, action, depth):
        step, child = sc.step(action.cpu().numpy(), depth.cpu().numpy())
        out = dm.RecurrentFnOutput(value=t(step["value"], torch.float32),
                                   action_values=t(step["action_values"], torch.float32),
                                   invalid_actions=t(step["invalid_actions"], torch.bool),
                                   terminal_outcome=t(step["terminal_outcome"], torch.int8),
                                   to_play=t(step["to_play"], torch.int32))
        return out, t(child, torch.int32)

    inv = sc.invalid_actions if sc.invalid_actions is not None else np.zeros_like(r["prior_logits"], bool)
    rule = (functools.partial(update_posterior_prefix_cdf, kappa=kappa, fallback_policy_samples=samples)
            if sc.prefix_cdf else functools.partial(update_posterior, kappa=kappa, policy_samples=samples))
    out = dm.dirichlet_thompson_policy((), sc.rng_key, root=root, recurrent_fn=recurrent,
                                       num_simulations=sc.num_simulations, invalid_actions=t(inv, torch.bool),
                                       posterior_update=rule, max_depth=sc.max_depth,
                                       policy_samples=sc.policy_samples)
    torch.cuda.synchronize()
    return types.SimpleNamespace(tree=NumpyTree(out.search_tree), action=out.action.cpu().numpy(),
                                 action_weights=out.action_weights.cpu().numpy())
