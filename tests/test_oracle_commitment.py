"""Action commitment restated on the CPU: the power-temperature sampler's
statistics, the argmax tie rules and the commitment policy's branches."""

import numpy as np

from oracle import oracle as O


def test_posterior_sample_action_follows_the_power_temperature_policy():
    # dirichlet_q_search.py:89-116: P(a) is proportional to p(a)^(1/T) over
    # the legal actions with positive policy
    B = 40000
    p = np.array([0.1, 0.0, 0.3, 0.6, 0.2], np.float32)
    legal = np.array([1, 1, 1, 0, 1], bool)
    for T in (1.0, 1.0 / 3.0):
        acts = O.commit_action("sample", O.PRNGKey(5), np.tile(p, (B, 1)), np.tile(legal, (B, 1)), T)
        freq = np.bincount(acts, minlength=5) / B
        w = np.where(legal & (p > 0), p.astype(np.float64) ** (1.0 / T), 0.0)
        np.testing.assert_allclose(freq, w / w.sum(), atol=0.01)


def test_posterior_sample_action_falls_back_to_legal_actions():
    B = 20000
    p = np.zeros((B, 4), np.float32)
    legal = np.tile(np.array([0, 1, 1, 0], bool), (B, 1))
    freq = np.bincount(O.commit_action("sample", O.PRNGKey(6), p, legal), minlength=4) / B
    np.testing.assert_allclose(freq, [0, 0.5, 0.5, 0], atol=0.015)


def test_posterior_best_action_tie_rules():
    policy = np.array([[0.2, 0.4, 0.4, 0.0], [0.9, np.nan, 0.1, np.nan], [0.3, 0.5, 0.2, 0.0]], np.float32)
    legal = np.array([[1, 1, 1, 1], [1, 1, 1, 1], [0, 0, 0, 0]], bool)
    assert O.commit_action("argmax", None, policy, legal).tolist() == [1, 1, 0]


def test_commitment_policy_branches():
    A = 4
    alpha = np.array([[[2, 3], [4, 1], [1, 2], [1, 1]]] * 3, np.float32)
    sampled = np.array([[0.5, 0.25, 0.25, 0.0]] * 3, np.float32)
    legal = np.array([[1, 1, 1, 0]] * 3, bool)
    evidence = np.array([[1, 1, 0, 0]] * 3, bool)
    q_out = np.full((3, A), -1, np.int8)
    v_out = np.array([-1, 1, -1], np.int8)
    action = np.array([0, 2, 0], np.int32)
    mc = O.commitment_policy(sampled, action, alpha, q_out, v_out, legal, evidence, search_evidence=True,
                             numerical=False)
    # support = legal actions with evidence: {0, 1}; sampled renormalised there
    np.testing.assert_allclose(mc[0], [2 / 3, 1 / 3, 0, 0], rtol=1e-6)
    # a categorical root commits the one-hot of its search action, but action
    # 2 is outside the support: the support's uniform fallback remains
    np.testing.assert_allclose(mc[1], [0.5, 0.5, 0, 0], rtol=1e-6)
    num = O.commitment_policy(sampled, action, alpha, q_out, v_out, legal, evidence, search_evidence=True,
                              numerical=True)
    est = O.prefix_cdf(alpha[:1], ~np.array([[1, 1, 0, 0]], bool), q_out[:1])
    np.testing.assert_array_equal(num[0], est.policy[0])
    np.testing.assert_array_equal(num[1], mc[1])  # categorical root: not a Q21 row
