"""Writes the committed golden fixtures of this directory from the oracle.

    python tests/golden/make_golden.py

The reference (pure JAX) cannot run here, so these vectors are the oracle's
outputs on seeded inputs: the oracle itself is pinned against the
reference's assertions and published known answers by
tests/test_oracle_pins.py and tests/test_oracle_scenarios.py.  The fixtures
freeze those outputs: tests/test_golden.py checks that the oracle still
reproduces them bit for bit, and tests/test_gpu_golden.py checks the CUDA
path against them without running the oracle.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

TREE_FIELDS = ("parents", "children_index", "node_to_play", "node_categorical_outcome", "node_payload",
               "edge_categorical_outcome", "edge_payload", "node_value_priors", "node_value_alpha", "edge_alpha",
               "invalid_actions")

# (name, lanes, simulations, prefix_cdf, terminal_prob, env seed, key seed, samples, kappa)
SEARCH_CASES = (
    ("prefix_terminal", 12, 14, True, 0.08, 4, 11, 8, 1.0),
    ("mc_kappa4", 12, 14, False, 0.0, 5, 12, 8, 4.0),
)

ESTIMATOR_LANES, ESTIMATOR_ACTIONS = 9, 82


def search_case(name, B, N, prefix, terminal_prob, seed, key_seed, samples, kappa) -> dict:
    from oracle import oracle as O

    env = O.synth_params(seed=seed, terminal_prob=terminal_prob)
    out = O.search_synthetic(env, B, O.PRNGKey(key_seed), N,
                             O.Rule(prefix_cdf=prefix, kappa=kappa, samples=samples),
                             max_depth=N, policy_samples=samples)
    d = {f"{name}.{f}": np.asarray(getattr(out.search_tree, f)) for f in TREE_FIELDS}
    d[f"{name}.action_weights"] = out.action_weights
    d[f"{name}.action"] = out.action
    d[f"{name}.unsafe_updates"] = np.array(out.unsafe_updates, np.int64)
    return d


def estimator_inputs():
    rng = np.random.default_rng(2024)
    B, A = ESTIMATOR_LANES, ESTIMATOR_ACTIONS
    alpha = np.exp(rng.uniform(-5, 6, (B, A, 2))).astype(np.float32)
    alpha[2] = 1e-3           # a degenerate lane (density guard)
    alpha[3, 0] = 1e-8        # a clipped half range
    invalid = rng.uniform(size=(B, A)) < 0.3
    invalid[7] = True         # no legal action
    cat = np.where(rng.uniform(size=(B, A)) < 0.1, rng.integers(0, 2, (B, A)), -1).astype(np.int8)
    cat[:2] = -1
    return alpha, invalid, cat


def estimator_case() -> dict:
    from oracle import oracle as O

    alpha, invalid, cat = estimator_inputs()
    r = O.prefix_cdf(alpha, invalid, cat, half_width=10)
    d = {f"prefix_cdf.{f}": np.asarray(getattr(r, f)) for f in r._fields}
    key = np.array([0x2545F491, 0x4F6CDD1D], np.uint32)
    d["posterior_best_policy.policy"] = O.posterior_best_policy(key, alpha, invalid, 8, cat)
    d["thompson_sample.action"] = O.thompson_sample(key, alpha, invalid, cat)
    return d


def generate() -> dict:
    d = {}
    for case in SEARCH_CASES:
        d.update(search_case(*case))
    d.update(estimator_case())
    return d


def main():
    path = os.path.join(HERE, "oracle_vectors.npz")
    np.savez_compressed(path, **generate())
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
