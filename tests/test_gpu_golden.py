"""The CUDA path against the committed golden vectors (no oracle run)."""

import functools
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden  # noqa: E402

pytestmark = pytest.mark.gpu

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oracle_vectors.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(FIXTURE)


@pytest.mark.parametrize("case", make_golden.SEARCH_CASES, ids=[c[0] for c in make_golden.SEARCH_CASES])
def test_search_matches_golden(cuda, golden, case):
    from scacchi_b200 import dirichlet_mctx as dm
    from scacchi_b200 import random as R
    from scacchi_b200.synthetic import SyntheticGame, SyntheticGameConfig

    name, B, N, prefix, terminal_prob, seed, key_seed, samples, kappa = case
    game = SyntheticGame(SyntheticGameConfig(seed=seed, terminal_prob=terminal_prob))
    rule = (functools.partial(dm.update_posterior_prefix_cdf, kappa=kappa, fallback_policy_samples=samples)
            if prefix else functools.partial(dm.update_posterior, kappa=kappa, policy_samples=samples))
    stats = torch.zeros(6, dtype=torch.int64, device="cuda")
    out = dm.dirichlet_thompson_policy((), R.PRNGKey(key_seed), root=game.root(B), recurrent_fn=game,
                                       num_simulations=N, posterior_update=rule, max_depth=N,
                                       policy_samples=samples, stats=stats)
    torch.cuda.synchronize()
    for f in make_golden.TREE_FIELDS:
        want = golden[f"{name}.{f}"]
        got = getattr(out.search_tree, f).cpu().numpy()
        assert np.array_equal(got.astype(want.dtype), want), f
    assert np.array_equal(out.action_weights.cpu().numpy(), golden[f"{name}.action_weights"])
    assert np.array_equal(out.action.cpu().numpy(), golden[f"{name}.action"])
    if prefix:
        assert int(stats[2]) == int(golden[f"{name}.unsafe_updates"])


def test_estimators_match_golden(cuda, golden):
    from scacchi_b200.dirichlet_mctx import binary_posterior_best_policy_prefix_quadrature as q
    from scacchi_b200.dirichlet_mctx.action_selection import posterior_best_policy, thompson_sample

    alpha, invalid, cat = make_golden.estimator_inputs()
    t = lambda x, dt: torch.as_tensor(np.asarray(x)).cuda().to(dt)
    a, inv, c = t(alpha, torch.float32), t(invalid, torch.bool), t(cat, torch.int8)
    r = q(a, inv, c, half_width=10)
    for f in r._fields:
        want = golden[f"prefix_cdf.{f}"]
        assert np.array_equal(getattr(r, f).cpu().numpy().astype(want.dtype), want, equal_nan=True), f
    key = np.array([0x2545F491, 0x4F6CDD1D], np.uint32)
    pol = posterior_best_policy(key, a, inv, 8, categorical_outcome=c)
    assert np.array_equal(pol.cpu().numpy(), golden["posterior_best_policy.policy"])
    act = thompson_sample(key, a, inv, categorical_outcome=c)
    assert np.array_equal(act.cpu().numpy(), golden["thompson_sample.action"])
