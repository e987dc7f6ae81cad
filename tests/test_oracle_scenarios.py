"""The oracle reproduces the tree-semantics assertions of the reference tests."""

import numpy as np
import pytest

from oracle import oracle as O
from tests import oracle_backend
from tests.scenarios import SCENARIOS


@pytest.mark.parametrize("sc", SCENARIOS, ids=[s.name for s in SCENARIOS])
def test_scenario(sc):
    sc.check(oracle_backend.run(sc))


def test_zero_simulation_policy_is_one_thompson_draw():
    # tests/test_dirichlet_q_search.py:868-908: with no simulations the
    # root policy is one Thompson draw under the policy key.
    sc = [s for s in SCENARIOS if s.name == "zero_simulations"][0]
    out = oracle_backend.run(sc)
    _, policy_key = O.split(sc.rng_key)
    sampled = O.sample_dirichlet(policy_key, sc.root["action_values"][0])
    util = sampled[:, 1] - sampled[:, 0]
    util = np.where(sc.invalid_actions[0], -np.inf, util)
    expected = int(np.argmax(util))
    assert out.action[0] == expected
    assert np.array_equal(out.action_weights[0], np.eye(3, dtype=np.float32)[expected])
