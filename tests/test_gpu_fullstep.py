"""The metric's workloads through make_search, pinned against the oracle.

Hex 9x9, 8192 lanes x 256 simulations (tree capacity 257), the reference's
random-init AZDirichletNet (6 x 128, zero-initialised output heads:
network.py:395-458) evaluating every leaf on the tcgen05 tower, exact
terminal certificates, roots after 0-20 uniform random legal moves; the
guarded prefix-CDF estimator (kappa 1, 8-sample Monte Carlo fallback) and
the 64-sample Thompson population.  With zero heads the tower's outputs are
one constant for every board (logits 0, alpha = c0 * softmax(0) with c0 =
3.1), which the test asserts; three lanes (first, middle, last) then rerun
on the oracle (the C restatement of the search driven by the Hex
restatement and that constant evaluator, at the lanes' places in the
8192-lane batch).  Every tree field, every expanded node's record and every
PosteriorTargets field of those lanes must match bit for bit
(play_search.py:435-548, dirichlet_q_search.py:43-76, search.py:189-251).
"""

import numpy as np
import pytest
import torch

from oracle import hex_ref as H

pytestmark = pytest.mark.gpu

LANES, SIMS = 8192, 256
SAMPLED = (0, LANES // 2, LANES - 1)
ROOT_KEY, SEARCH_KEY = 3, 11


def _prefix_cfg():
    from scacchi_b200.types import (DirichletThompsonSearchConfig, NumericalPosteriorUpdateConfig,
                                    PosteriorUpdateConfig, PosteriorUpdateKind, RootPolicySupport)

    return DirichletThompsonSearchConfig(
        num_simulations=SIMS, max_depth=SIMS, root_policy_support=RootPolicySupport.search_evidence,
        policy_target_temperature=1.0,
        posterior_update=PosteriorUpdateConfig(
            kind=PosteriorUpdateKind.numerical,
            numerical=NumericalPosteriorUpdateConfig(kappa=1.0, half_width=10, tail_scale=8.0, min_half_range=6.0,
                                                     max_half_range=11.0, fallback_policy_samples=8,
                                                     fallback_policy_sample_chunk_size=32)))


def _population_cfg():
    from scacchi_b200.types import (DirichletThompsonSearchConfig, MonteCarloPosteriorUpdateConfig,
                                    PosteriorUpdateConfig, PosteriorUpdateKind, RootPolicySupport)

    return DirichletThompsonSearchConfig(
        num_simulations=SIMS, max_depth=SIMS, root_policy_support=RootPolicySupport.search_evidence,
        policy_target_temperature=1.0,
        posterior_update=PosteriorUpdateConfig(
            kind=PosteriorUpdateKind.monte_carlo,
            monte_carlo=MonteCarloPosteriorUpdateConfig(kappa=1.0, policy_samples=64, policy_sample_chunk_size=32)))


@pytest.fixture(scope="module")
def workload(cuda):
    """Roots, the random-init tower and its constant outputs."""
    from scacchi_b200 import random as R
    from scacchi_b200.hex import HexGame
    from scacchi_b200.network import AZDirichletNet, init_params

    game = HexGame(9)
    state = game.random_roots(LANES, R.PRNGKey(ROOT_KEY), 0, 20)
    net = AZDirichletNet(init_params(0, he_all_layers=False))
    logits, av, aq = net(state.observation)
    torch.cuda.synchronize()
    # zero heads: one constant output for every board
    assert not logits.any()
    av0, aq0 = av[0].clone(), aq[0].clone()
    assert torch.equal(av, av0.expand_as(av)) and torch.equal(aq, aq0.expand_as(aq))
    np.testing.assert_allclose(av0.cpu().numpy(), 1.55, rtol=1e-6)
    np.testing.assert_allclose(aq0.cpu().numpy(), 1.55, rtol=1e-6)
    return game, state, net, av0.cpu().numpy(), aq0.cpu().numpy()


def test_roots_match_the_restated_sampler(workload):
    from oracle import oracle as O

    game, state, _, _, _ = workload
    rec = state.record.cpu().numpy()
    for lane in SAMPLED:
        want = H.random_root(9, O.PRNGKey(ROOT_KEY), lane, 0, 20)
        assert np.array_equal(rec[lane, :H.RECORD_BYTES], want.record()), lane


def _oracle_lane(lane, rec, legal, av0, aq0, rule, policy_samples):
    """The oracle's search of one lane of the batch with the constant evaluator."""
    from oracle import oracle as O

    A = aq0.shape[0]
    board = H.HexBoard.from_record(rec)
    root_term = (int(board.rewards()[board.current_player()]) + 1) // 2 if board.terminated else -1
    inv = ~legal[None]
    root = dict(prior_logits=np.zeros((1, A), np.float32), value=av0[None].copy(), action_values=aq0[None].copy(),
                terminal_outcome=np.array([root_term], np.int8), to_play=np.array([board.current_player()], np.int32),
                embedding=rec[None, :H.RECORD_BYTES])

    def recurrent(actions, parent_emb):
        outs = [H.step_outputs(r, a) for r, a in zip(parent_emb, actions)]
        n = len(outs)
        step = dict(value=np.repeat(av0[None], n, 0), action_values=np.repeat(aq0[None], n, 0),
                    invalid_actions=np.stack([o["invalid"] for o in outs]),
                    terminal_outcome=np.array([o["terminal"] for o in outs], np.int8),
                    to_play=np.array([o["to_play"] for o in outs], np.int32))
        return step, np.stack([o["record"] for o in outs])

    return O.dirichlet_thompson_policy(
        np.asarray(O.PRNGKey(SEARCH_KEY), np.uint32), root=root, recurrent_fn=recurrent, num_simulations=SIMS,
        invalid_actions=inv, rule=rule, max_depth=SIMS, policy_samples=policy_samples, lane_offset=lane,
        total_batch=LANES)


TREE_FIELDS = ("parents", "children_index", "node_to_play", "node_categorical_outcome", "node_payload",
               "edge_categorical_outcome", "edge_payload", "node_value_priors", "node_value_alpha", "edge_alpha",
               "invalid_actions")


def _check_lanes(workload, cfg, rule, policy_samples, numerical):
    from oracle import oracle as O
    from scacchi_b200 import _lib
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import make_evaluator, make_search

    game, state, net, av0, aq0 = workload
    search = make_search(game, make_evaluator(net), cfg, keep_output=True)
    targets = search(state, R.PRNGKey(SEARCH_KEY))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0 and _lib.tower_error() == 0
    tree = search.last_output.search_tree
    rec = state.record.cpu().numpy()
    legal_all = state.legal_action_mask.cpu().numpy()
    solved = 0
    for lane in SAMPLED:
        want = _oracle_lane(lane, rec[lane], legal_all[lane], av0, aq0, rule, policy_samples)
        for f in TREE_FIELDS:
            got = getattr(tree, f)[lane].cpu().numpy()
            ref = getattr(want.search_tree, f)[0]
            assert np.array_equal(got.astype(ref.dtype), ref), (lane, f)
        parents = want.search_tree.parents[0]
        expanded = parents >= 0
        expanded[0] = True
        emb = tree.embedding_[lane].cpu().numpy()[..., :H.RECORD_BYTES]
        assert np.array_equal(emb[expanded], want.search_tree.embeddings[0][expanded]), lane
        assert expanded.sum() > 1
        # root readout and target packing
        s = want.search_tree.summary()
        legal = legal_all[lane:lane + 1]
        if numerical:
            policy_target, _ = O.root_readout(want.action_weights, s, legal, search_evidence=True, temperature=1.0,
                                              rule=rule)
        else:
            policy_target = want.action_weights
        ref_t = O.pack_targets(s, policy_target, legal, want.action)
        md = targets.metadata
        got_t = dict(policy=targets.prediction.policy, alpha_q=targets.prediction.alpha_q,
                     alpha_v=targets.prediction.alpha_v, mask=md.mask, q_supervision_selected=md.q_supervision.selected,
                     q_supervision_pair_weight=md.q_supervision.pair_weight,
                     q_positive_evidence_action=md.q_positive_evidence_action,
                     q_positive_policy_action=md.q_positive_policy_action, search_action=md.search_action,
                     q_target_kind=md.q_target_kind, q_target_weight=md.q_target_weight,
                     q_target_outcome=md.q_target_outcome, q_target_distance=md.q_target_distance,
                     v_target_kind=md.v_target_kind, v_target_weight=md.v_target_weight,
                     v_target_outcome=md.v_target_outcome, v_target_distance=md.v_target_distance)
        for k, v in got_t.items():
            g = v[lane:lane + 1].cpu().numpy()
            r = np.asarray(ref_t[k])
            assert np.array_equal(g.astype(r.dtype), r), (lane, k)
        solved += int((want.search_tree.node_categorical_outcome[0] >= 0).any())
    return solved


def test_full_step_prefix_cdf_matches_oracle(workload):
    """The full Hex 9x9 search step (8192 lanes x 256 simulations, prefix-CDF
    estimator) on sampled lanes."""
    from oracle import oracle as O

    _check_lanes(workload, _prefix_cfg(), O.Rule(prefix_cdf=True, kappa=1.0, samples=8), 8, numerical=True)


def test_population_step_matches_oracle(workload):
    """The same step with the 64-sample Thompson-population estimator (the
    per-GPU shard of the 8-GPU lane-sharded workload)."""
    from oracle import oracle as O

    _check_lanes(workload, _population_cfg(), O.Rule(prefix_cdf=False, kappa=1.0, samples=64), 64, numerical=False)
