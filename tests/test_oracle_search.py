"""Consistency of the oracle's whole-search driver with its own pieces."""

import numpy as np

from oracle import oracle as O


def test_root_policy_of_synthetic_search_is_the_population_on_the_root_summary():
    env = O.synth_params(seed=0, terminal_prob=0.0)
    B, N = 24, 12
    out = O.search_synthetic(env, B, O.PRNGKey(0), N, O.Rule(prefix_cdf=True, kappa=1.0, samples=8),
                             max_depth=N, policy_samples=8)
    s = out.search_tree.summary()
    inv = O.synthetic_root(env, B)["invalid_actions"]
    pol = O.posterior_best_policy(O.split(O.PRNGKey(0))[1], s["alpha"], inv, 8, s["q_categorical_outcome"])
    assert np.array_equal(pol, out.action_weights)


def test_lane_ranges_reproduce_the_full_batch():
    env = O.synth_params(seed=4, terminal_prob=0.05)
    rule = O.Rule(prefix_cdf=True, kappa=1.0, samples=8)
    full = O.search_synthetic(env, 12, O.PRNGKey(1), 10, rule)
    part = O.search_synthetic(env, 12, O.PRNGKey(1), 10, rule, lanes=(4, 9))
    for f in ("parents", "children_index", "edge_payload", "edge_alpha", "node_value_alpha", "node_payload"):
        assert np.array_equal(getattr(full.search_tree, f)[4:9], getattr(part.search_tree, f)), f
    assert np.array_equal(full.action_weights[4:9], part.action_weights)


def test_python_driven_loop_matches_c_loop():
    """oracle.dirichlet_thompson_policy (Python loop, synthetic recurrent fn)
    equals oracle.search_synthetic (loop in C)."""
    env = O.synth_params(seed=2, terminal_prob=0.1)
    B, N = 10, 9
    rule = O.Rule(prefix_cdf=True, kappa=1.0, samples=8)
    root = O.synthetic_root(env, B)
    a = O.dirichlet_thompson_policy(O.PRNGKey(3), root=root, recurrent_fn=lambda act, emb: O.synthetic_recurrent(
        env, act, emb), num_simulations=N, invalid_actions=root["invalid_actions"], rule=rule, max_depth=N,
        policy_samples=8)
    b = O.search_synthetic(env, B, O.PRNGKey(3), N, rule, max_depth=N, policy_samples=8)
    for f in ("parents", "children_index", "edge_payload", "edge_alpha", "node_value_alpha", "node_payload"):
        assert np.array_equal(getattr(a.search_tree, f), getattr(b.search_tree, f)), f
    assert np.array_equal(a.action_weights, b.action_weights)
