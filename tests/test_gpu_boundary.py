"""make_search on the reference's toy environments (tests/test_play.py:72-155,
236-365, 734-866 of the reference), on the CUDA path.

Expected values the reference computes with jax.random come from the
oracle's threefry-exact restatement (same keys, same batch layout)."""

from typing import NamedTuple

import numpy as np
import pytest
import torch

from scacchi_b200.play_search import TARGET_CATEGORICAL, TARGET_PAD

pytestmark = pytest.mark.gpu


class ToyState(NamedTuple):
    observation: torch.Tensor
    legal_action_mask: torch.Tensor
    current_player: torch.Tensor
    rewards: torch.Tensor
    terminated: torch.Tensor


class ToyEnv:
    """_ToySearchEnv: observation + 1, everything else unchanged."""

    def step(self, state, action):
        return state._replace(observation=state.observation + 1.0)


class TerminalToyEnv:
    """_TerminalToySearchEnv: every move wins for the mover."""

    def step(self, state, action):
        actor = state.current_player.long()
        rewards = 2.0 * torch.nn.functional.one_hot(actor, 2).to(state.observation.dtype) - 1.0
        return ToyState(observation=state.observation + 1.0,
                        legal_action_mask=torch.zeros_like(state.legal_action_mask),
                        current_player=(1 - state.current_player), rewards=rewards,
                        terminated=torch.ones_like(state.terminated))


ALPHA_V = [2.0, 3.0]
ALPHA_Q = [[3.0, 1.0], [1.0, 4.0], [2.0, 2.0]]


def toy_evaluator(obs):
    from scacchi_b200.play_search import EvaluatorOutput

    B = obs.shape[0]
    dev = obs.device
    return EvaluatorOutput(logits=torch.zeros((B, 3), device=dev),
                           alpha_v=torch.tensor(ALPHA_V, device=dev).expand(B, 2).contiguous(),
                           alpha_q=torch.tensor(ALPHA_Q, device=dev).expand(B, 3, 2).contiguous())


def toy_state():
    dev = "cuda"
    return ToyState(observation=torch.zeros((2, 1), device=dev),
                    legal_action_mask=torch.tensor([[True, True, False], [False, True, True]], device=dev),
                    current_player=torch.zeros(2, dtype=torch.int32, device=dev),
                    rewards=torch.zeros((2, 2), device=dev),
                    terminated=torch.zeros(2, dtype=torch.bool, device=dev))


def config(num_simulations, kind="monte_carlo", samples=1, chunk=2, max_depth=None):
    from scacchi_b200.types import (DirichletThompsonSearchConfig, MonteCarloPosteriorUpdateConfig,
                                    NumericalPosteriorUpdateConfig, PosteriorUpdateConfig, PosteriorUpdateKind,
                                    SearchConfig, SearchKind)

    return SearchConfig(kind=SearchKind.dirichlet_thompson, dirichlet_thompson=DirichletThompsonSearchConfig(
        num_simulations=num_simulations, max_depth=max_depth,
        posterior_update=PosteriorUpdateConfig(
            kind=PosteriorUpdateKind(kind),
            monte_carlo=MonteCarloPosteriorUpdateConfig(policy_samples=samples, policy_sample_chunk_size=chunk),
            numerical=NumericalPosteriorUpdateConfig(fallback_policy_samples=samples,
                                                     fallback_policy_sample_chunk_size=chunk))))


def policy_q_supervision():
    from scacchi_b200.types import QActionSet, QPairReduction, QSupervisionConfig

    return QSupervisionConfig(action_set=QActionSet.positive_posterior_policy_or_solved,
                              reduction=QPairReduction.mean_over_selected_state_action_pairs)


def test_prior_only_search_preserves_rng_and_targets(cuda):
    # tests/test_play.py:236-293
    from oracle import oracle as O
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import make_search

    state = toy_state()
    key = R.PRNGKey(17)
    out = make_search(ToyEnv(), toy_evaluator, config(0, samples=1), policy_q_supervision())(state, key)
    torch.cuda.synchronize()
    _, policy_key = O.split(O.PRNGKey(17))
    legal = state.legal_action_mask.cpu().numpy()
    alpha_q = np.broadcast_to(np.array(ALPHA_Q, np.float32), (2, 3, 2)).copy()
    expected_action = O.thompson_sample(policy_key, alpha_q, ~legal)
    expected_policy = np.eye(3, dtype=np.float32)[expected_action]
    m = out.metadata
    assert np.array_equal(out.prediction.policy.cpu().numpy(), expected_policy)
    assert np.array_equal(out.prediction.alpha_q.cpu().numpy(), alpha_q)
    assert np.array_equal(out.prediction.alpha_v.cpu().numpy(), np.array([ALPHA_V] * 2, np.float32))
    assert np.array_equal(m.q_supervision.selected.cpu().numpy(), expected_policy.astype(bool))
    assert np.array_equal(m.q_supervision.pair_weight.cpu().numpy(), expected_policy)
    assert np.array_equal(m.search_action.cpu().numpy(), expected_action)
    assert m.mask.cpu().numpy().all()


def test_numerical_update_drives_q21_root_target(cuda):
    # tests/test_play.py:296-365
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import make_search

    state = toy_state()
    key = R.PRNGKey(91)
    native = make_search(ToyEnv(), toy_evaluator, config(0, samples=8), policy_q_supervision())(state, key)
    numerical = make_search(ToyEnv(), toy_evaluator, config(0, "numerical", samples=8),
                            policy_q_supervision())(state, key)
    assert not torch.equal(numerical.prediction.policy, native.prediction.policy)
    assert torch.equal(native.metadata.q_supervision.selected, native.prediction.policy > 0)
    assert torch.equal(numerical.metadata.q_supervision.selected, numerical.prediction.policy > 0)
    assert torch.equal(numerical.metadata.q_supervision.pair_weight,
                       numerical.metadata.q_supervision.selected.to(numerical.prediction.policy.dtype))


def test_one_unsafe_q21_root_lane_does_not_change_safe_lane(cuda):
    # tests/test_play.py:736-804
    from oracle import oracle as O
    from scacchi_b200.dirichlet_mctx.tree import SearchSummary
    from scacchi_b200.play_search import dirichlet_root_policy_readout
    from scacchi_b200.types import DirichletThompsonSearchConfig, PosteriorUpdateConfig, PosteriorUpdateKind

    native = torch.tensor([[0.25, 0.50, 0.25], [0.50, 0.25, 0.25]], device="cuda")
    alpha = np.array([[[2.0, 3.0], [4.0, 1.0], [1.0, 2.0]], [[1e-5, 1.0], [2.0, 1.0], [1.0, 3.0]]], np.float32)
    cat = np.full((2, 3), -1, np.int8)
    summary = SearchSummary(visit_counts=torch.ones((2, 3), device="cuda"), alpha=torch.from_numpy(alpha).cuda(),
                            value_alpha=torch.ones((2, 2), device="cuda"),
                            q_categorical_outcome=torch.from_numpy(cat).cuda(),
                            q_categorical_distance=torch.zeros((2, 3), dtype=torch.int32, device="cuda"),
                            v_categorical_outcome=torch.full((2,), -1, dtype=torch.int8, device="cuda"),
                            v_categorical_distance=torch.zeros(2, dtype=torch.int32, device="cuda"))
    cfg = DirichletThompsonSearchConfig(posterior_update=PosteriorUpdateConfig(kind=PosteriorUpdateKind.numerical))
    readout = dirichlet_root_policy_readout(native, summary, torch.ones((2, 3), dtype=torch.bool, device="cuda"),
                                            cfg).cpu().numpy()
    est = O.prefix_cdf(alpha, np.zeros((2, 3), bool), cat)
    assert est.tail_range_clipped.tolist() == [False, True]
    np.testing.assert_allclose(readout[0], est.policy[0], atol=1e-6)
    assert np.array_equal(readout[1], native[1].cpu().numpy())


@pytest.mark.parametrize("kind", ["monte_carlo", "numerical"])
def test_tree_search_builds_legal_targets(cuda, kind):
    # tests/test_play.py:807-866
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import make_search

    state = toy_state()
    out = make_search(ToyEnv(), toy_evaluator, config(4, kind, samples=1, max_depth=2))(state, R.PRNGKey(23))
    p, m = out.prediction, out.metadata
    legal = state.legal_action_mask
    assert p.policy.shape == legal.shape and p.alpha_v.shape == (2, 2) and p.alpha_q.shape == (2, 3, 2)
    assert torch.allclose(p.policy.sum(-1), torch.ones(2, device="cuda"))
    assert (p.policy[~legal] == 0).all()
    expected_selected = m.q_positive_evidence_action | (m.q_target_kind == TARGET_CATEGORICAL)
    assert torch.equal(m.q_supervision.selected, expected_selected)
    assert torch.equal(m.q_supervision.pair_weight, expected_selected.to(p.policy.dtype))
    assert m.mask.all()
    assert legal.gather(1, m.search_action.long()[:, None]).all()


def test_exports_categorical_root_and_q_targets(cuda):
    # tests/test_play.py:869-906
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import make_search
    from scacchi_b200.types import DirichletThompsonSearchConfig, SearchConfig, SearchKind

    state = toy_state()
    cfg = SearchConfig(kind=SearchKind.dirichlet_thompson,
                       dirichlet_thompson=DirichletThompsonSearchConfig(num_simulations=4))
    out = make_search(TerminalToyEnv(), toy_evaluator, cfg)(state, R.PRNGKey(29))
    p, m = out.prediction, out.metadata
    batch = torch.arange(2, device="cuda")
    action = m.search_action.long()
    assert torch.equal(p.policy, torch.nn.functional.one_hot(action, 3).to(p.policy.dtype))
    assert (m.q_target_kind[batch, action] == TARGET_CATEGORICAL).all()
    assert (m.q_target_outcome[batch, action] == 1).all()
    assert (m.q_target_distance[batch, action] == 1).all()
    assert (m.v_target_kind == TARGET_CATEGORICAL).all()
    assert (m.v_target_outcome == 1).all()
    assert (m.v_target_distance == 1).all()
    assert (m.q_target_kind[~state.legal_action_mask] == TARGET_PAD).all()
