"""Tree-semantics scenarios restated from the reference's own tests.

Each scenario is the root, recurrent function and assertions of one test in
``tests/test_dirichlet_q_search.py`` / ``tests/test_dirichlet_mctx_categorical.py``
of Francesco215/Scacchi (cited per scenario).  The same scenario runs on the
C oracle (CPU tests) and through the CUDA search (GPU tests); ``check`` gets a
numpy view of the finished search with the reference's attribute names.

Embeddings are an int32 depth counter, as in the reference tests.
"""

from __future__ import annotations

import dataclasses
from typing import Callable

import numpy as np

NO_OUTCOME = -1
NO_DISTANCE = -1


def prng_key(seed: int) -> np.ndarray:
    return np.array([0, seed], np.uint32)


def make_root(action_values, *, value=None, to_play=0, terminal_outcome=NO_OUTCOME):
    action_values = np.asarray(action_values, np.float32)
    if action_values.ndim == 2:
        action_values = action_values[None]
    B, A, O = action_values.shape
    if value is None:
        value = np.ones((B, O), np.float32)
    return dict(
        prior_logits=np.zeros((B, A), np.float32),
        value=np.asarray(value, np.float32).reshape(B, O),
        action_values=action_values,
        terminal_outcome=np.full(B, terminal_outcome, np.int8),
        to_play=np.full(B, to_play, np.int32),
        embedding=np.zeros(B, np.int32),
    )


def constant_step(*, num_actions, value, action_values=None, to_play, terminal_outcome=NO_OUTCOME,
                  invalid_actions=None):
    """_constant_recurrent_fn, tests/test_dirichlet_q_search.py:101-137."""
    if invalid_actions is None:
        invalid_actions = (False,) * num_actions
    if action_values is None:
        action_values = (value,) * num_actions

    def step(action, depth):
        B = action.shape[0]
        out = dict(
            value=np.broadcast_to(np.asarray(value, np.float32), (B, len(value))).copy(),
            action_values=np.broadcast_to(np.asarray(action_values, np.float32),
                                          (B, num_actions, len(value))).copy(),
            invalid_actions=np.broadcast_to(np.asarray(invalid_actions, bool), (B, num_actions)).copy(),
            terminal_outcome=np.full(B, terminal_outcome, np.int8),
            to_play=np.full(B, to_play, np.int32),
        )
        return out, depth + 1

    return step


@dataclasses.dataclass
class Scenario:
    name: str
    root: dict
    step: Callable
    num_simulations: int
    invalid_actions: np.ndarray | None = None
    max_depth: int | None = None
    policy_samples: int = 0
    rng_key: np.ndarray = dataclasses.field(default_factory=lambda: prng_key(0))
    prefix_cdf: bool = False
    check: Callable = lambda out: None


def _close(a, b, **kw):
    np.testing.assert_allclose(np.asarray(a, np.float64), np.asarray(b, np.float64), rtol=1e-5, atol=1e-6, **kw)


def _first_leaf_check(out):
    tree = out.tree
    s = tree.summary()
    _close(s["alpha"], [[[6.0, 2.0], [1.0, 9.0]]])
    assert np.array_equal(tree.edge_payload[:, 0], [[1, 0]])
    _close(tree.node_value_alpha[:, 0], [[2.0, 1.2]])
    assert np.array_equal(s["visit_counts"], [[1.0, 0.0]])
    assert int(tree.children_index[0, 0, 0]) == 1


def _depth_cutoff_check(out):
    tree = out.tree
    s = tree.summary()
    assert np.array_equal(s["visit_counts"], [[4.0]])
    _close(s["alpha"], [[[3.0, 1.0]]])
    _close(tree.node_value_alpha[:, 0], [[2.0, 1.0]])
    assert int(tree.children_index[0, 0, 0]) == 1
    assert np.array_equal(tree.parents[0], [-1, 0, -1, -1, -1])


def _terminal_child_check(out):
    tree = out.tree
    assert int(tree.children_index[0, 0, 1]) == 1
    assert tree.node_categorical_outcome[0, 1] != NO_OUTCOME
    assert np.all(tree.children_index[0, 1] == -1)
    assert np.array_equal(tree.parents[0], [-1, 0, -1, -1])
    s = tree.summary()
    assert np.array_equal(s["visit_counts"], [[0.0, 0.0]])
    _close(s["alpha"], [[[1.0, 1.0], [1.0, 1.0]]])
    assert np.array_equal(s["q_categorical_outcome"], [[NO_OUTCOME, 1]])
    assert np.array_equal(s["q_categorical_distance"], [[NO_DISTANCE, 1]])
    _close(tree.node_value_alpha[0, 0], [0.8, 1.2])
    _close(tree.node_value_priors[0, 1], [4.0, 2.0])
    assert tree.node_categorical_outcome[0, 0] == 1
    assert tree.node_payload[0, 0] == 1


def _chain_step(terminal_depth):
    """chain_recurrent_fn, tests/test_dirichlet_q_search.py:618-640."""

    def step(action, depth):
        child = depth + 1
        B = child.shape[0]
        terminal = child >= terminal_depth
        return dict(
            value=np.ones((B, 2), np.float32),
            action_values=np.ones((B, 1, 2), np.float32),
            invalid_actions=terminal[:, None].copy(),
            terminal_outcome=np.where(terminal, 1, NO_OUTCOME).astype(np.int8),
            to_play=np.zeros(B, np.int32),
        ), child

    return step


def _chain_check(out):
    tree = out.tree
    d = 5
    assert tree.node_categorical_outcome[0, d] != NO_OUTCOME
    assert np.array_equal(tree.parents[0, 1:d + 1], np.arange(d))
    assert np.array_equal(tree.children_index[0, :d, 0], np.arange(1, d + 1))
    s = tree.summary()
    assert s["visit_counts"][0, 0] == 0
    assert s["q_categorical_outcome"][0, 0] == 1
    assert s["q_categorical_distance"][0, 0] == d
    assert tree.edge_categorical_outcome[0, d - 1, 0] == 1
    assert tree.edge_payload[0, d - 1, 0] == 1


def _terminal_root_check(out):
    assert np.array_equal(out.tree.edge_payload[:, 0], [[0]])


def _bottom_up_step(action, depth):
    """tests/test_dirichlet_q_search.py:691-717."""
    B = action.shape[0]
    nxt = depth + 1
    first = nxt == 1
    value = np.where(first[:, None], np.array([[2.0, 5.0]]), np.array([[7.0, 3.0]])).astype(np.float32)
    return dict(
        value=value,
        action_values=np.ones((B, 3, 2), np.float32),
        invalid_actions=np.broadcast_to(np.array([True, False, True]), (B, 3)).copy(),
        terminal_outcome=np.full(B, NO_OUTCOME, np.int8),
        to_play=np.ones(B, np.int32),
    ), nxt


def _bottom_up_check(out):
    tree = out.tree
    s = tree.summary()
    _close(s["alpha"][0, 2], [4.6, 3.0])
    assert np.array_equal(s["visit_counts"], [[0.0, 0.0, 2.0]])
    rc = int(tree.children_index[0, 0, 2])
    assert rc == 1
    assert int(tree.children_index[0, rc, 1]) == 2
    _close(tree.edge_alpha[0, rc, 1], [7.0, 3.0])
    assert int(tree.edge_payload[0, rc, 1]) == 1
    _close(tree.node_value_alpha[0, rc], [3.0, 4.6])
    _close(tree.node_value_alpha[:, 0], [[2.2, 5.0 / 3.0]])


def _persistent_check(out):
    tree = out.tree
    s = tree.summary()
    _close(s["alpha"], [[[4.0, 1.0]]])
    assert np.array_equal(s["visit_counts"], [[3.0]])
    _close(tree.node_value_alpha[:, 0], [[16.0 / 7.0, 1.0]])
    assert int(tree.children_index[0, 0, 0]) == 1


def _hetero_check(out):
    assert np.array_equal(out.action, [0, 1])
    _close(out.action_weights.sum(-1), [1.0, 1.0])
    inv = np.array([[False, True], [True, False]])
    assert np.all(out.action_weights[inv] == 0.0)
    assert np.array_equal(out.tree.summary()["visit_counts"], [[2.0, 0.0], [0.0, 2.0]])


def _zero_sim_check(out):
    tree = out.tree
    assert np.array_equal(tree.edge_alpha[:, 0], [[[1.0, 4.0], [4.0, 1.0], [2.0, 2.0]]])
    assert not tree.edge_payload[:, 0].any()
    assert not tree.node_payload.any()
    assert np.all(tree.children_index == -1)
    assert out.action_weights.sum() == 1.0
    assert out.action_weights[0, out.action[0]] == 1.0


def _expand_terminal_step(action, depth):
    """_ExpandEnv + _expand_evaluator with a terminated root state, the
    native expand fn of tests/test_dirichlet_q_search.py:257-306: player 0
    won, the child (player 1) sees a certified loss."""
    B = action.shape[0]
    return dict(
        value=np.broadcast_to(np.array([2.0, 6.0], np.float32), (B, 2)).copy(),
        action_values=np.broadcast_to(np.array([[3.0, 1.0], [1.0, 3.0]], np.float32), (B, 2, 2)).copy(),
        invalid_actions=np.broadcast_to(np.array([False, True]), (B, 2)).copy(),
        terminal_outcome=np.zeros(B, np.int8),
        to_play=np.ones(B, np.int32),
    ), depth + 1


def _expand_terminal_check(out):
    tree = out.tree
    s = tree.summary()
    assert s["q_categorical_outcome"][0, 0] == 1
    assert s["v_categorical_outcome"][0] == 1
    assert np.array_equal(out.action_weights, [[1.0, 0.0]])
    assert np.array_equal(s["alpha"][0, 0], [1.0, 1.0])
    child = int(tree.children_index[0, 0, 0])
    assert np.array_equal(tree.node_value_priors[0, child], [2.0, 6.0])


SCENARIOS = [
    Scenario(
        "first_leaf_replaces_q_fallback",  # test_dirichlet_q_search.py:352-380
        make_root([[9.0, 1.0], [1.0, 9.0]], to_play=0),
        constant_step(num_actions=2, value=(2.0, 6.0), to_play=1),
        num_simulations=1, invalid_actions=np.array([[False, True]]), max_depth=4, check=_first_leaf_check),
    Scenario(
        "repeated_depth_cutoff",  # test_dirichlet_q_search.py:518-543
        make_root([[1.0, 1.0]], to_play=0),
        constant_step(num_actions=1, value=(3.0, 1.0), to_play=0),
        num_simulations=4, max_depth=1, check=_depth_cutoff_check),
    Scenario(
        "terminal_child_short_circuits",  # test_dirichlet_q_search.py:545-593
        make_root([[1.0, 1.0], [1.0, 1.0]], to_play=0),
        constant_step(num_actions=2, value=(4.0, 2.0), to_play=1, terminal_outcome=0,
                      invalid_actions=(True, True)),
        num_simulations=3, invalid_actions=np.array([[True, False]]), max_depth=6, check=_terminal_child_check),
    Scenario(
        "default_max_depth_chain",  # test_dirichlet_q_search.py:595-669
        make_root([[1.0, 1.0]]),
        _chain_step(5),
        num_simulations=6, max_depth=6, check=_chain_check),
    Scenario(
        "terminal_root_does_not_search",  # test_dirichlet_q_search.py:671-688
        make_root([[1.0, 1.0]], terminal_outcome=0),
        constant_step(num_actions=1, value=(2.0, 1.0), to_play=0),
        num_simulations=1, invalid_actions=np.array([[False]]), check=_terminal_root_check),
    Scenario(
        "bottom_up_repair_players",  # test_dirichlet_q_search.py:690-749
        make_root([[1.0, 1.0], [1.0, 1.0], [1.0, 1.0]], to_play=0),
        _bottom_up_step,
        num_simulations=2, invalid_actions=np.array([[True, True, False]]), max_depth=2, check=_bottom_up_check),
    Scenario(
        "persistent_tree",  # test_dirichlet_q_search.py:751-776
        make_root([[1.0, 1.0]], to_play=0),
        constant_step(num_actions=1, value=(4.0, 1.0), to_play=0),
        num_simulations=3, max_depth=1, rng_key=prng_key(11), check=_persistent_check),
    Scenario(
        "heterogeneous_root_masks",  # test_dirichlet_q_search.py:911-948
        make_root([[[2.0, 1.0], [1.0, 2.0]], [[1.0, 3.0], [3.0, 1.0]]]),
        constant_step(num_actions=2, value=(2.0, 4.0), to_play=1),
        num_simulations=2, invalid_actions=np.array([[False, True], [True, False]]), max_depth=2,
        policy_samples=4, rng_key=prng_key(9), check=_hetero_check),
    Scenario(
        "zero_simulations",  # test_dirichlet_q_search.py:868-908
        make_root([[[1.0, 4.0], [4.0, 1.0], [2.0, 2.0]]]),
        constant_step(num_actions=3, value=(1.0, 1.0), to_play=1),
        num_simulations=0, invalid_actions=np.array([[False, False, True]]), rng_key=prng_key(17),
        check=_zero_sim_check),
    Scenario(
        "expand_publishes_exact_terminal",  # test_dirichlet_q_search.py:257-306
        make_root([[[1.0, 1.0], [1.0, 1.0]]]),
        _expand_terminal_step,
        num_simulations=2, invalid_actions=np.array([[False, True]]), policy_samples=8,
        check=_expand_terminal_check),
]


def _alternating_chain_step(terminal_depth):
    """recurrent_fn of tests/test_dirichlet_mctx_categorical.py:203-227 with
    binary outcomes (win index 1): the terminal child is a certified loss for
    its player and the players alternate by depth."""

    def step(action, depth):
        child = depth + 1
        B = child.shape[0]
        td = np.broadcast_to(np.asarray(terminal_depth), (B,))
        terminal = child >= td
        return dict(
            value=np.ones((B, 2), np.float32),
            action_values=np.ones((B, 1, 2), np.float32),
            invalid_actions=terminal[:, None].copy(),
            terminal_outcome=np.where(terminal, 0, NO_OUTCOME).astype(np.int8),
            to_play=(child % 2).astype(np.int32),
        ), child

    return step


def _terminal_chain_check(out):
    # tests/test_dirichlet_mctx_categorical.py:242-272 (win index 2 -> 1)
    tree = out.tree
    assert np.array_equal(tree.node_categorical_outcome[0, :4], [1, 0, 1, 0])
    assert np.array_equal(tree.node_payload[0, :4], [3, 2, 1, 0])
    assert np.array_equal(tree.edge_categorical_outcome[0, :3, 0], [1, 0, 1])
    assert np.array_equal(tree.edge_payload[0, :3, 0], [3, 2, 1])
    assert np.array_equal(tree.parents[0], [-1, 0, 1, 2, -1, -1, -1, -1])
    assert out.action[0] == 0
    assert np.array_equal(out.action_weights, [[1.0]])
    s = tree.summary()
    assert s["v_categorical_outcome"][0] == 1
    assert s["v_categorical_distance"][0] == 3
    assert s["q_categorical_outcome"][0, 0] == 1
    assert s["q_categorical_distance"][0, 0] == 3


def _frozen_lane_check(out):
    # tests/test_dirichlet_mctx_categorical.py:325-342
    tree = out.tree
    assert np.array_equal(tree.node_categorical_outcome[:, 0], [1, 1])
    assert np.array_equal(tree.node_payload[:, 0], [1, 3])
    assert np.array_equal(tree.parents[0], [-1, 0, -1, -1, -1, -1])
    assert np.array_equal(tree.parents[1], [-1, 0, 1, 2, -1, -1])
    assert np.array_equal(out.action_weights, np.ones((2, 1)))


SCENARIOS += [
    Scenario(
        "terminal_chain_perspective_and_distance",  # test_dirichlet_mctx_categorical.py:203-272
        make_root([[1.0, 1.0]]),
        _alternating_chain_step(3),
        num_simulations=7, invalid_actions=np.array([[False]]), max_depth=7, policy_samples=4,
        rng_key=prng_key(11), check=_terminal_chain_check),
    Scenario(
        "solved_lane_stays_frozen",  # test_dirichlet_mctx_categorical.py:274-342
        make_root([[[1.0, 1.0]], [[1.0, 1.0]]]),
        _alternating_chain_step(np.array([1, 3])),
        num_simulations=5, invalid_actions=np.zeros((2, 1), bool), max_depth=5, policy_samples=4,
        rng_key=prng_key(17), check=_frozen_lane_check),
]
