"""Reference tree-semantics scenarios through the CUDA search, checked with the
reference's assertions and bit-for-bit against the oracle."""

import numpy as np
import pytest

from tests.scenarios import SCENARIOS

pytestmark = pytest.mark.gpu

FIELDS = ("parents", "children_index", "node_to_play", "node_categorical_outcome", "node_payload",
          "edge_categorical_outcome", "edge_payload", "node_value_priors", "node_value_alpha", "edge_alpha",
          "invalid_actions")


@pytest.mark.parametrize("prefix", [False, True], ids=["mc", "prefix_cdf"])
@pytest.mark.parametrize("sc", SCENARIOS, ids=[s.name for s in SCENARIOS])
def test_scenario_matches_reference_and_oracle(cuda, sc, prefix):
    from tests import gpu_backend, oracle_backend
    from oracle import oracle as O
    import dataclasses

    sc = dataclasses.replace(sc, prefix_cdf=prefix)
    got = gpu_backend.run(sc)
    if not prefix:
        sc.check(got)
    want = oracle_backend.run(sc, O.Rule(prefix_cdf=prefix, samples=32, kappa=4.0))
    for f in FIELDS:
        a = np.asarray(getattr(got.tree, f))
        b = np.asarray(getattr(want.tree, f))
        assert a.shape == b.shape, f
        assert np.array_equal(a, b), f"{f}: cuda {a} oracle {b}"
    assert np.array_equal(got.action, want.action)
    assert np.array_equal(got.action_weights, want.action_weights)
